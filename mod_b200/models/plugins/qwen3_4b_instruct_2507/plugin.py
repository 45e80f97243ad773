"""Qwen3-4B-Instruct-2507 plugin (counterpart of ``pio/models/qwen3_4b_instruct_2507/plugin.py``)."""
from ....api.engine_plugin import EnginePlugin


class Qwen3_4B_Instruct_2507_Plugin(EnginePlugin):
    preset = "qwen3-4b-instruct-2507"
    display_name = "Qwen3-4B-Instruct-2507"
    family = "Qwen"
    architecture = "Qwen3 Transformer"
    size = "4B"
    modalities = ('text',)
    # the 2507 Instruct release is the non-thinking variant: replies start directly with the answer
    thinking_default = False


def create_qwen3_4b_instruct_2507_plugin():
    return Qwen3_4B_Instruct_2507_Plugin()
