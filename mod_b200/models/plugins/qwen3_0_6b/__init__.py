from .plugin import Qwen3_0_6B_Plugin, create_qwen3_0_6b_plugin  # noqa: F401
