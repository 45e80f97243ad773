from .plugin import Qwen3_Coder_30B_Plugin, create_qwen3_coder_30b_plugin  # noqa: F401
