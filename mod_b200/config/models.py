"""Model configurations, one dataclass per family, HF ``config.json`` compatible.

The reference keeps one config class per model with two incompatible styles
(dataclasses for 30B/Next/VL/GLM, ``__init__`` overrides for 0.6B/4B;
``pio/common/config/model_config_base.py:9-60``,
``pio/models/qwen3_0_6b/config.py:4-22``).  Here every family derives from
:class:`ModelConfig`, and :func:`from_hf_dict` maps HF keys onto it.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional


@dataclass
class ModelConfig:
    """Decoder-only transformer (Qwen3 dense/MoE, GLM)."""

    model_type: str = "qwen3"
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    partial_rotary_factor: float = 1.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = True
    qk_norm: bool = True
    attention_bias: bool = False
    hidden_act: str = "silu"            # "silu" (SwiGLU MLP) or "gelu" (GLM-style 4h MLP)
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    shared_expert_intermediate_size: int = 0
    decoder_sparse_step: int = 1
    # hybrid (Qwen3-Next): per-layer "linear_attention" / "full_attention"
    layer_types: Optional[List[str]] = None
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel_dim: int = 4
    attn_output_gate: bool = False
    name: str = ""
    torch_dtype: str = "bfloat16"

    # ------------------------------------------------------------------ derived
    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def layer_type(self, i: int) -> str:
        if self.layer_types:
            return self.layer_types[i]
        return "full_attention"

    def num_params(self) -> int:
        H, L = self.hidden_size, self.num_hidden_layers
        n = self.vocab_size * H * (1 if self.tie_word_embeddings else 2) + H
        for i in range(L):
            if self.layer_type(i) == "full_attention":
                qo = self.q_size * (2 if self.attn_output_gate else 1)
                n += H * (qo + 2 * self.kv_size) + self.q_size * H
            else:
                kd = self.linear_num_key_heads * self.linear_key_head_dim
                vd = self.linear_num_value_heads * self.linear_value_head_dim
                n += H * (2 * kd + 2 * vd + 2 * self.linear_num_value_heads) + vd * H
                n += (2 * kd + vd) * self.linear_conv_kernel_dim
            if self.is_moe:
                n += H * self.num_experts + self.num_experts * 3 * H * self.moe_intermediate_size
                if self.shared_expert_intermediate_size:
                    n += 3 * H * self.shared_expert_intermediate_size + H
            else:
                mult = 3 if self.hidden_act == "silu" else 2
                n += mult * H * self.intermediate_size
            n += 2 * H
        return n

    def active_params(self) -> int:
        if not self.is_moe:
            return self.num_params()
        H = self.hidden_size
        dense = self.num_params() - self.num_hidden_layers * self.num_experts * 3 * H * self.moe_intermediate_size
        return dense + self.num_hidden_layers * self.num_experts_per_tok * 3 * H * self.moe_intermediate_size

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)

    def to_json(self, path: str) -> None:
        with open(path, "w") as f:
            json.dump(self.to_dict(), f, indent=2)

    def validate(self) -> None:
        assert self.num_attention_heads % self.num_key_value_heads == 0, "GQA needs heads % kv_heads == 0"
        assert self.hidden_size % 8 == 0
        if self.is_moe:
            assert 0 < self.num_experts_per_tok <= self.num_experts
            assert self.moe_intermediate_size > 0
        if self.layer_types:
            assert len(self.layer_types) == self.num_hidden_layers


@dataclass
class VisionConfig:
    """ViT encoder of Qwen3-VL style models (patch embed, 2-D RoPE, 2x2 merger)."""

    hidden_size: int = 1024
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    intermediate_size: int = 4096
    patch_size: int = 16
    in_channels: int = 3
    spatial_merge_size: int = 2
    out_hidden_size: int = 2048
    layer_norm_eps: float = 1e-6
    image_mean: tuple = (0.5, 0.5, 0.5)
    image_std: tuple = (0.5, 0.5, 0.5)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


@dataclass
class VLConfig:
    text: ModelConfig = field(default_factory=ModelConfig)
    vision: VisionConfig = field(default_factory=VisionConfig)
    image_token_id: int = 151655
    model_type: str = "qwen3_vl"
    name: str = ""

    def validate(self) -> None:
        self.text.validate()
        assert self.vision.out_hidden_size == self.text.hidden_size


_HF_ALIASES = {"n_layer": "num_hidden_layers", "n_head": "num_attention_heads", "n_embd": "hidden_size"}


def from_hf_dict(d: Dict[str, Any]) -> ModelConfig:
    """Builds a :class:`ModelConfig` from an HF ``config.json`` dict."""
    known = {f.name for f in dataclasses.fields(ModelConfig)}
    kw = {}
    for k, v in d.items():
        k = _HF_ALIASES.get(k, k)
        if k in known:
            kw[k] = v
    if "head_dim" not in d and "hidden_size" in d and "num_attention_heads" in d:
        kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
    if d.get("shared_expert_intermediate_size"):
        kw["shared_expert_intermediate_size"] = d["shared_expert_intermediate_size"]
    cfg = ModelConfig(**kw)
    cfg.validate()
    return cfg


def load_config(path: str) -> ModelConfig:
    with open(path) as f:
        return from_hf_dict(json.load(f))
