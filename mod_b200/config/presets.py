"""Named model shapes.

The full-size presets are the architectures the benchmarks are quoted on
(Qwen3-0.6B, Qwen3-8B, Qwen3-30B-A3B, Qwen3-VL, Qwen3-Next); the ``tiny-*``
presets keep every structural feature (GQA, QK-norm, MoE top-k, hybrid layer
pattern, vision merger) at shapes small enough for CPU tests.  The reference
ships one plugin per model (``pio/models/*``); its Qwen3-0.6B config is at
``pio/models/qwen3_0_6b/config.py:11-18`` and the 30B MoE one at
``pio/models/qwen3_coder_30b/config.py:19-31``.
"""
from __future__ import annotations

import copy
from typing import Callable, Dict, Union

from .models import ModelConfig, VisionConfig, VLConfig


def qwen3_0_6b() -> ModelConfig:
    return ModelConfig(name="qwen3-0.6b", hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, tie_word_embeddings=True)


def qwen3_4b() -> ModelConfig:
    return ModelConfig(name="qwen3-4b-instruct-2507", hidden_size=2560, intermediate_size=9728,
                       num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                       max_position_embeddings=262144, rope_theta=5_000_000.0, tie_word_embeddings=True)


def qwen3_8b() -> ModelConfig:
    return ModelConfig(name="qwen3-8b", hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=128, tie_word_embeddings=False)


def qwen3_30b_a3b() -> ModelConfig:
    return ModelConfig(name="qwen3-30b-a3b", model_type="qwen3_moe", hidden_size=2048, intermediate_size=6144,
                       num_hidden_layers=48, num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                       num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768, norm_topk_prob=True,
                       tie_word_embeddings=False, max_position_embeddings=131072)


def qwen3_next() -> ModelConfig:
    L = 48
    return ModelConfig(name="qwen3-next", model_type="qwen3_next", hidden_size=2048, intermediate_size=5120,
                       num_hidden_layers=L, num_attention_heads=16, num_key_value_heads=2, head_dim=256,
                       partial_rotary_factor=0.25, num_experts=512, num_experts_per_tok=10,
                       moe_intermediate_size=512, shared_expert_intermediate_size=512, norm_topk_prob=True,
                       layer_types=["linear_attention" if (i + 1) % 4 else "full_attention" for i in range(L)],
                       linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128,
                       linear_value_head_dim=128, linear_conv_kernel_dim=4, attn_output_gate=True,
                       tie_word_embeddings=False, max_position_embeddings=262144)


def glm_4_7_flash() -> ModelConfig:
    # Plugin-parity model: GQA attention with qkv bias and a GELU 4h MLP, the
    # architecture the reference's GLM plugin actually runs
    # (pio/models/glm_4_7_flash/model.py:186-306).
    return ModelConfig(name="glm-4.7-flash", model_type="glm", hidden_size=2048, intermediate_size=8192,
                       num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=4, head_dim=128,
                       qk_norm=False, attention_bias=True, hidden_act="gelu", rope_theta=10000.0,
                       vocab_size=151552, tie_word_embeddings=False)


def qwen3_vl() -> VLConfig:
    text = ModelConfig(name="qwen3-vl-text", hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, tie_word_embeddings=True)
    vis = VisionConfig(hidden_size=1024, num_hidden_layers=24, num_attention_heads=16, intermediate_size=4096,
                       patch_size=16, spatial_merge_size=2, out_hidden_size=2048)
    return VLConfig(text=text, vision=vis, name="qwen3-vl")


# ---------------------------------------------------------------- tiny shapes
def tiny_dense() -> ModelConfig:
    return ModelConfig(name="tiny-dense", vocab_size=512, hidden_size=256, intermediate_size=512,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                       tie_word_embeddings=True)


def tiny_moe() -> ModelConfig:
    return ModelConfig(name="tiny-moe", model_type="qwen3_moe", vocab_size=512, hidden_size=256,
                       intermediate_size=512, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=128, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=128,
                       tie_word_embeddings=False)


def tiny_next() -> ModelConfig:
    return ModelConfig(name="tiny-next", model_type="qwen3_next", vocab_size=512, hidden_size=256,
                       intermediate_size=512, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=128, partial_rotary_factor=0.5, num_experts=16, num_experts_per_tok=4,
                       moe_intermediate_size=128, shared_expert_intermediate_size=128,
                       layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
                       linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=64,
                       linear_value_head_dim=64, attn_output_gate=True, tie_word_embeddings=False)


def tiny_glm() -> ModelConfig:
    c = glm_4_7_flash()
    c.name, c.vocab_size, c.hidden_size, c.intermediate_size = "tiny-glm", 512, 256, 1024
    c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads = 2, 4, 2
    return c


def tiny_vl() -> VLConfig:
    text = tiny_dense()
    text.name = "tiny-vl-text"
    vis = VisionConfig(hidden_size=128, num_hidden_layers=2, num_attention_heads=2, intermediate_size=256,
                       patch_size=16, spatial_merge_size=2, out_hidden_size=256)
    return VLConfig(text=text, vision=vis, name="tiny-vl", image_token_id=500)


PRESETS: Dict[str, Callable[[], Union[ModelConfig, VLConfig]]] = {
    "qwen3-0.6b": qwen3_0_6b,
    "qwen3-4b-instruct-2507": qwen3_4b,
    "qwen3-8b": qwen3_8b,
    "qwen3-30b-a3b": qwen3_30b_a3b,
    "qwen3-coder-30b": qwen3_30b_a3b,
    "qwen3-next": qwen3_next,
    "qwen3-coder-next": qwen3_next,
    "qwen3-vl": qwen3_vl,
    "qwen3-vl-2b": qwen3_vl,
    "glm-4.7-flash": glm_4_7_flash,
    "tiny-dense": tiny_dense,
    "tiny-moe": tiny_moe,
    "tiny-next": tiny_next,
    "tiny-glm": tiny_glm,
    "tiny-vl": tiny_vl,
}


def get_preset(name: str):
    key = name.lower().replace("_", "-")
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return copy.deepcopy(PRESETS[key]())
