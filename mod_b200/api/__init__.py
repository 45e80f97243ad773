"""Plugin API: interfaces, plugin manager, backends, model factory."""
from .interfaces import (HardwareBackendInterface, ModelPluginInterface, PluginMetadata, PluginType,  # noqa: F401
                         TextModelPluginInterface, VisionLanguagePluginInterface)
from .manager import (ModelFactory, PluginManager, SecondaryPlugin, SecondaryPluginManager,  # noqa: F401
                      SecondaryPluginType, create_model, get_plugin_manager, get_secondary_plugin_manager)
