"""GLM-4.7-Flash plugin (counterpart of ``pio/models/glm_4_7_flash/plugin.py``)."""
from ....api.engine_plugin import EnginePlugin


class GLM_4_7_Flash_Plugin(EnginePlugin):
    preset = "glm-4.7-flash"
    display_name = "GLM-4.7-Flash"
    family = "GLM"
    architecture = "GLM transformer (GQA, qkv bias, GELU MLP)"
    size = "flash"
    modalities = ('text',)


def create_glm_4_7_flash_plugin():
    return GLM_4_7_Flash_Plugin()
