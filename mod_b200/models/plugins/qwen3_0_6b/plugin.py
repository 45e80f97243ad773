"""Qwen3-0.6B plugin (counterpart of ``pio/models/qwen3_0_6b/plugin.py:20-178``)."""
from ....api.engine_plugin import EnginePlugin


class Qwen3_0_6B_Plugin(EnginePlugin):
    preset = "qwen3-0.6b"
    display_name = "Qwen3-0.6B"
    family = "Qwen"
    architecture = "Qwen3 Transformer"
    size = "0.6B"
    modalities = ('text',)
    # Qwen3 dense checkpoints are hybrid-thinking models: a chat reply opens with a <think> block by default
    thinking_default = True


def create_qwen3_0_6b_plugin():
    return Qwen3_0_6B_Plugin()
