"""Qwen3-Coder-30B plugin (counterpart of ``pio/models/qwen3_coder_30b/plugin.py``)."""
from ....api.engine_plugin import EnginePlugin


class Qwen3_Coder_30B_Plugin(EnginePlugin):
    preset = "qwen3-30b-a3b"
    display_name = "Qwen3-Coder-30B"
    family = "Qwen"
    architecture = "Qwen3 MoE Transformer"
    size = "30B-A3B"
    modalities = ('text',)
    # Qwen coder checkpoints are trained for fill-in-the-middle with these markers (complete_code)
    fim_tokens = ("<|fim_prefix|>", "<|fim_suffix|>", "<|fim_middle|>")


def create_qwen3_coder_30b_plugin():
    return Qwen3_Coder_30B_Plugin()
