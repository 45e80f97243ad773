"""Qwen3-Coder-Next plugin (counterpart of ``pio/models/qwen3_coder_next/plugin.py``)."""
from ....api.engine_plugin import EnginePlugin


class Qwen3_Coder_Next_Plugin(EnginePlugin):
    preset = "qwen3-next"
    display_name = "Qwen3-Coder-Next"
    family = "Qwen"
    architecture = "Qwen3-Next hybrid gated DeltaNet + gated attention MoE"
    size = "80B-A3B"
    modalities = ('text',)
    fim_tokens = ("<|fim_prefix|>", "<|fim_suffix|>", "<|fim_middle|>")
    # long-context hybrid model: int8 weight-only projections (512 experts) and chunked prefill so a 32k-token
    # prompt alternates with running decodes instead of stalling them
    gpu_runtime_defaults = {"quantization": "int8", "prefill_chunk": 8192}


def create_qwen3_coder_next_plugin():
    return Qwen3_Coder_Next_Plugin()
