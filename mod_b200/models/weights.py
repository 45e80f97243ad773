"""Weight containers and random initialisation.

Weights are kept in the fused layouts the kernels consume:

* ``qkv``      [(Hq + 2*Hkv) * D (+ Hq*D output gate), H]  (q, k, v[, gate] rows)
* ``gate_up``  [2*I, H]                                   (gate rows, then up rows)
* ``w13``      [E * 2*I, H]   experts stacked, each [gate; up]
* ``w2``       [E * H, I]     experts stacked

HF checkpoints are mapped onto these by :mod:`mod_b200.io.hf_loader`.
Random initialisation is N(0, 0.02) from a seeded generator, norms are ones:
the rule the benchmarks use for synthetic weights.  The reference never
initialises its Linear weights (``pio/core/engine/backend.py:695-702``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from ..config.models import ModelConfig


@dataclass
class AttnWeights:
    qkv: torch.Tensor
    o: torch.Tensor
    q_norm: Optional[torch.Tensor] = None
    k_norm: Optional[torch.Tensor] = None
    qkv_bias: Optional[torch.Tensor] = None
    o_bias: Optional[torch.Tensor] = None


@dataclass
class DeltaNetWeights:
    """Gated DeltaNet (Qwen3-Next linear attention)."""
    in_qkvz: torch.Tensor        # [2*Kd + 2*Vd, H]  (q, k, v, z)
    in_ba: torch.Tensor          # [2*Hv, H]         (beta logits, decay logits)
    conv: torch.Tensor           # [2*Kd + Vd, kernel] depthwise causal conv
    A_log: torch.Tensor          # [Hv]
    dt_bias: torch.Tensor        # [Hv]
    norm: torch.Tensor           # [Dv]  gated RMSNorm weight
    out: torch.Tensor            # [H, Vd]


@dataclass
class MLPWeights:
    gate_up: Optional[torch.Tensor] = None   # SwiGLU [2I, H]
    up: Optional[torch.Tensor] = None        # GELU MLP [I, H]
    down: Optional[torch.Tensor] = None      # [H, I]
    up_bias: Optional[torch.Tensor] = None
    down_bias: Optional[torch.Tensor] = None


@dataclass
class MoEWeights:
    router: torch.Tensor                     # [E, H]
    w13: torch.Tensor                        # [E*2I, H]
    w2: torch.Tensor                         # [E*H, I]
    shared: Optional[MLPWeights] = None
    shared_gate: Optional[torch.Tensor] = None   # [1, H]
    # expert-parallel sharding: this rank owns experts [e_lo, e_hi)
    e_lo: int = 0
    e_hi: int = 0


@dataclass
class LayerWeights:
    kind: str                                # "full_attention" | "linear_attention"
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    attn: Optional[AttnWeights] = None
    delta: Optional[DeltaNetWeights] = None
    mlp: Optional[MLPWeights] = None
    moe: Optional[MoEWeights] = None


@dataclass
class ModelWeights:
    embed: torch.Tensor
    layers: List[LayerWeights]
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    extra: Dict[str, torch.Tensor] = field(default_factory=dict)

    def tensors(self):
        """Yields (name, tensor) for every weight (used by save/load and byte counts)."""
        yield "embed", self.embed
        yield "final_norm", self.final_norm
        if self.lm_head is not self.embed:
            yield "lm_head", self.lm_head
        for i, L in enumerate(self.layers):
            for part in ("attn", "delta", "mlp", "moe"):
                obj = getattr(L, part)
                if obj is None:
                    continue
                for k, v in vars(obj).items():
                    if isinstance(v, torch.Tensor):
                        yield f"layers.{i}.{part}.{k}", v
                    elif isinstance(v, MLPWeights):
                        for k2, v2 in vars(v).items():
                            if isinstance(v2, torch.Tensor):
                                yield f"layers.{i}.{part}.{k}.{k2}", v2
            yield f"layers.{i}.in_norm", L.in_norm
            yield f"layers.{i}.post_norm", L.post_norm

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for _, t in self.tensors())


class _Init:
    def __init__(self, device, dtype, seed: int, std: float = 0.02):
        self.device, self.dtype, self.std = device, dtype, std
        gdev = device if torch.device(device).type == "cuda" else "cpu"
        self.gen = torch.Generator(device=gdev)
        self.gen.manual_seed(seed)

    def normal(self, *shape) -> torch.Tensor:
        t = torch.empty(*shape, device=self.device, dtype=self.dtype)
        t.normal_(0.0, self.std, generator=self.gen)
        return t

    def ones(self, *shape) -> torch.Tensor:
        return torch.ones(*shape, device=self.device, dtype=self.dtype)

    def zeros(self, *shape) -> torch.Tensor:
        return torch.zeros(*shape, device=self.device, dtype=self.dtype)

    def expert_normal(self, out: torch.Tensor, seed: int, layer: int, expert: int, which: int) -> None:
        """Fills ``out`` from a generator keyed by (seed, layer, expert, which), so an
        expert's weights do not depend on how experts are sharded across ranks."""
        self.egen = getattr(self, "egen", None) or torch.Generator(device=self.gen.device)
        self.egen.manual_seed(((seed * 1_000_003 + layer) * 4099 + expert) * 3 + which + 17)
        out.normal_(0.0, self.std, generator=self.egen)


def random_weights(cfg: ModelConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                   expert_range: Optional[tuple] = None, quantize: Optional[str] = None) -> ModelWeights:
    """N(0, 0.02) weights of the given architecture.

    ``expert_range=(lo, hi)`` materialises only experts [lo, hi) (expert
    parallelism).  Expert weights come from per-(layer, expert) generators and
    everything else from one sequential generator, so every rank of an
    expert-parallel group holds the same dense weights and the union of the
    shards equals the unsharded model.  ``quantize="int8"`` converts each layer's
    projections as soon as the layer exists, so the bf16 copy of the whole model
    is never held at once (a 77B-parameter model fits one GPU as int8).
    """
    cfg.validate()
    ini = _Init(device, dtype, seed)
    H, D = cfg.hidden_size, cfg.head_dim
    embed = ini.normal(cfg.vocab_size, H)
    layers: List[LayerWeights] = []
    for i in range(cfg.num_hidden_layers):
        kind = cfg.layer_type(i)
        L = LayerWeights(kind=kind, in_norm=ini.ones(H), post_norm=ini.ones(H))
        if kind == "full_attention":
            rows = cfg.q_size * (2 if cfg.attn_output_gate else 1) + 2 * cfg.kv_size
            L.attn = AttnWeights(qkv=ini.normal(rows, H), o=ini.normal(H, cfg.q_size))
            if cfg.qk_norm:
                L.attn.q_norm, L.attn.k_norm = ini.ones(D), ini.ones(D)
            if cfg.attention_bias:
                L.attn.qkv_bias = ini.zeros(rows)
                L.attn.o_bias = ini.zeros(H)
        else:
            kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
            vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
            hv = cfg.linear_num_value_heads
            L.delta = DeltaNetWeights(
                in_qkvz=ini.normal(2 * kd + 2 * vd, H), in_ba=ini.normal(2 * hv, H),
                conv=ini.normal(2 * kd + vd, cfg.linear_conv_kernel_dim),
                A_log=torch.log(torch.linspace(1.0, 16.0, hv, device=device)).to(torch.float32),
                dt_bias=torch.ones(hv, device=device, dtype=torch.float32),
                norm=ini.ones(cfg.linear_value_head_dim), out=ini.normal(H, vd))
        if cfg.is_moe:
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            lo, hi = expert_range if expert_range else (0, E)
            n = hi - lo
            w13 = torch.empty(n * 2 * I, H, device=device, dtype=dtype)
            w2 = torch.empty(n * H, I, device=device, dtype=dtype)
            for j, e in enumerate(range(lo, hi)):
                ini.expert_normal(w13[j * 2 * I:(j + 1) * 2 * I], seed, i, e, 0)
                ini.expert_normal(w2[j * H:(j + 1) * H], seed, i, e, 1)
            moe = MoEWeights(router=ini.normal(E, H), w13=w13, w2=w2, e_lo=lo, e_hi=hi)
            if cfg.shared_expert_intermediate_size:
                S = cfg.shared_expert_intermediate_size
                moe.shared = MLPWeights(gate_up=ini.normal(2 * S, H), down=ini.normal(H, S))
                moe.shared_gate = ini.normal(1, H)
            L.moe = moe
        else:
            I = cfg.intermediate_size
            if cfg.hidden_act == "silu":
                L.mlp = MLPWeights(gate_up=ini.normal(2 * I, H), down=ini.normal(H, I))
            else:
                L.mlp = MLPWeights(up=ini.normal(I, H), down=ini.normal(H, I), up_bias=ini.zeros(I),
                                   down_bias=ini.zeros(H))
        if quantize == "int8":
            from ..ops.quant import quantize_layer

            quantize_layer(L)
        elif quantize not in (None, "none"):
            raise ValueError(f"unknown quantization {quantize!r}")
        layers.append(L)
    final_norm = ini.ones(H)
    lm_head = embed if cfg.tie_word_embeddings else ini.normal(cfg.vocab_size, H)
    return ModelWeights(embed=embed, layers=layers, final_norm=final_norm, lm_head=lm_head)
