from .plugin import GLM_4_7_Flash_Plugin, create_glm_4_7_flash_plugin  # noqa: F401
