"""Qwen3-VL-2B plugin (counterpart of ``pio/models/qwen3_vl_2b/plugin.py``)."""
from ...vl import VisionLanguageEnginePlugin


class Qwen3_VL_2B_Plugin(VisionLanguageEnginePlugin):
    preset = "qwen3-vl"
    display_name = "Qwen3-VL-2B"
    family = "Qwen"
    architecture = "Qwen3-VL (ViT + LLM)"
    size = "2B"
    modalities = ('text', 'image')


def create_qwen3_vl_2b_plugin():
    return Qwen3_VL_2B_Plugin()
