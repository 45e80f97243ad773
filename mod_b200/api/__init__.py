"""Plugin API: interfaces, plugin manager, backends, model factory."""
from .interfaces import (HardwareBackendInterface, ModelPluginInterface, PluginMetadata, PluginType,  # noqa: F401
                         TextModelPluginInterface, VisionLanguagePluginInterface)
from .manager import (ModelFactory, PluginManager, SecondaryPluginManager, SecondaryPluginType,  # noqa: F401
                      create_model, get_plugin_manager)
