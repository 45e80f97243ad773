from .plugin import Qwen3_Coder_Next_Plugin, create_qwen3_coder_next_plugin  # noqa: F401
