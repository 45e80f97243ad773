"""int8 weight-only quantisation with per-output-channel scales.

``w ~= q * scale[:, None]`` with ``q = round(w / scale)`` in [-127, 127] and
``scale = max|w_row| / 127``.  The native GEMM (``linear_w8``) streams the
int8 rows, expands them to bf16 in shared memory and applies ``scale`` in the
epilogue, so weight bytes halve against bf16 while activations stay bf16.

The reference quantises per tensor and dequantises to fp32 before a plain
matmul (``pio/plugins/cuda/c_src/tensor_ops_cuda.cu:31-63, 475-478``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class Int8Weight:
    q: torch.Tensor        # int8 [N, K]
    scale: torch.Tensor    # f32 [N]

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    @property
    def dtype(self):
        return torch.int8

    def dequant(self, dtype=torch.bfloat16) -> torch.Tensor:
        return (self.q.float() * self.scale[:, None]).to(dtype)

    def to(self, device) -> "Int8Weight":
        return Int8Weight(self.q.to(device), self.scale.to(device))


def quantize_int8(w: torch.Tensor) -> Int8Weight:
    """Symmetric per-row int8 quantisation of a [N, K] weight."""
    wf = w.float()
    amax = wf.abs().amax(dim=1).clamp_min(1e-8)
    scale = amax / 127.0
    q = torch.round(wf / scale[:, None]).clamp_(-127, 127).to(torch.int8)
    return Int8Weight(q.contiguous(), scale.contiguous())


def is_int8(w) -> bool:
    return isinstance(w, Int8Weight)


def dense(w, dtype=torch.bfloat16) -> Optional[torch.Tensor]:
    """Plain tensor view of a weight (dequantised when int8)."""
    if w is None:
        return None
    return w.dequant(dtype) if isinstance(w, Int8Weight) else w


def quantize_layer(L, experts: bool = True, attention: bool = True, mlp: bool = True,
                   linear_attention: bool = True) -> None:
    """In place: the large projection matrices of one layer become :class:`Int8Weight`."""
    if attention and L.attn is not None:
        L.attn.qkv = quantize_int8(L.attn.qkv)
        L.attn.o = quantize_int8(L.attn.o)
    if linear_attention and L.delta is not None:
        L.delta.in_qkvz = quantize_int8(L.delta.in_qkvz)
        L.delta.out = quantize_int8(L.delta.out)
    if mlp and L.mlp is not None and L.mlp.gate_up is not None:
        L.mlp.gate_up = quantize_int8(L.mlp.gate_up)
        L.mlp.down = quantize_int8(L.mlp.down)
    if L.moe is not None:
        if experts:
            L.moe.w13 = quantize_int8(L.moe.w13)
            L.moe.w2 = quantize_int8(L.moe.w2)
        if mlp and L.moe.shared is not None:
            L.moe.shared.gate_up = quantize_int8(L.moe.shared.gate_up)
            L.moe.shared.down = quantize_int8(L.moe.shared.down)


def quantize_model(weights, experts: bool = True, attention: bool = True, mlp: bool = True,
                   linear_attention: bool = True):
    """In-place: replace the large projection matrices of every layer by
    :class:`Int8Weight`.  Embedding, LM head, norms, router and gates stay bf16."""
    for L in weights.layers:
        quantize_layer(L, experts, attention, mlp, linear_attention)
    return weights
