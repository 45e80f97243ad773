from .plugin import Qwen3_VL_2B_Plugin, create_qwen3_vl_2b_plugin  # noqa: F401
