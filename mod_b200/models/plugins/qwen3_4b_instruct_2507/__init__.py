from .plugin import Qwen3_4B_Instruct_2507_Plugin, create_qwen3_4b_instruct_2507_plugin  # noqa: F401
