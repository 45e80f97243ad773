"""Context-parallel prefill of one long prompt, handed to the serving engine.

A prompt of S tokens is cut into one contiguous chunk per rank of a process
group (ceil(S / N) tokens each, the last padded at its end, which causal
attention never lets a real token see).  Every rank runs the whole layer
stack on its own chunk: projections, norms, MLP / MoE locally (weights
replicated), attention across ranks with :func:`parallel.cp.ring_attention`
(K/V chunks passed around the ring) or :func:`parallel.cp.ulysses_attention`
(head <-> sequence all-to-all).  Activation memory and attention work per
rank are 1/N of a single-GPU prefill of the same prompt.

Afterwards the K/V chunks are all-gathered, so every rank holds the prompt's
full cache, and the last prompt token's logits give the first output token.
:meth:`engine.llm_engine.LLMEngine.generate_context_parallel` puts that cache
into the engine's paged KV pool and decodes from it with the normal
continuous-batching path (no recomputation of the prompt).

Baseline form: torch.distributed and fp32 torch math per chunk, so it runs on
any backend including gloo.  Attention-only decoders (dense or MoE); hybrid
DeltaNet models keep their single-rank chunked prefill.  The reference has no
long-context parallelism; its attention materialises the S x S scores
(``src/inference_pio/plugins/cpu/c_src/tensor_ops.c:544``).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..config.models import ModelConfig
from ..models import oracle as O
from ..models.weights import ModelWeights
from ..ops import reference as R
from .cp import ring_attention, ulysses_attention


def _attention(cfg: ModelConfig, aw, h: torch.Tensor, pos: torch.Tensor, mode: str, group):
    """h [c, H] (normed chunk) -> (attention output [c, H], k [c, Hkv, D] after QK-norm + RoPE, v)."""
    Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    c = h.shape[0]
    qkv = h @ O._f(aw.qkv).t()
    if aw.qkv_bias is not None:
        qkv = qkv + O._f(aw.qkv_bias)
    q = qkv[:, :Hq * D].reshape(c, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(c, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].reshape(c, Hkv, D)
    if aw.q_norm is not None:
        q = O.rms(q, O._f(aw.q_norm), cfg.rms_norm_eps)
        k = O.rms(k, O._f(aw.k_norm), cfg.rms_norm_eps)
    invf = R.inv_freq(cfg.rotary_dim, cfg.rope_theta, device=h.device)
    q = R.apply_rope(q, pos, invf, cfg.rotary_dim)
    k = R.apply_rope(k, pos, invf, cfg.rotary_dim)
    fn = ring_attention if mode == "ring" else ulysses_attention
    o = fn(q, k, v, causal=True, scale=D ** -0.5, group=group).float().reshape(c, Hq * D)
    if cfg.attn_output_gate:
        o = o * torch.sigmoid(qkv[:, (Hq + 2 * Hkv) * D:])
    y = o @ O._f(aw.o).t()
    if aw.o_bias is not None:
        y = y + O._f(aw.o_bias)
    return y, k, v


@torch.no_grad()
def cp_prefill(cfg: ModelConfig, w: ModelWeights, prompt: Sequence[int], group=None,
               mode: str = "ring") -> Tuple[torch.Tensor, List[torch.Tensor], List[torch.Tensor]]:
    """Collective over ``group`` (every rank passes the same prompt and weights).

    Returns (logits [V] of the last prompt token, K and V of every attention
    layer as [S, Hkv, D] fp32), identical on every rank."""
    if mode not in ("ring", "ulysses"):
        raise ValueError(f"context-parallel attention mode {mode!r} (ring | ulysses)")
    if any(L.kind != "full_attention" for L in w.layers):
        raise NotImplementedError("context-parallel prefill covers attention-only decoders")
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    dev = w.embed.device
    S = len(prompt)
    c = -(-S // world)
    ids = torch.tensor(list(prompt) + [0] * (c * world - S), device=dev)[rank * c:(rank + 1) * c]
    pos = torch.arange(rank * c, (rank + 1) * c, device=dev)
    eps = cfg.rms_norm_eps
    x = O._f(w.embed)[ids]                                               # [c, H]
    ks, vs = [], []
    for L in w.layers:
        y, k, v = _attention(cfg, L.attn, O.rms(x, O._f(L.in_norm), eps), pos, mode, group)
        x = x + y
        h = O.rms(x, O._f(L.post_norm), eps)[None]
        x = x + (O.moe_block(cfg, L.moe, h) if L.moe is not None else O.mlp_block(cfg, L.mlp, h))[0]
        ks.append(k)
        vs.append(v)
    owner = (S - 1) // c
    last = O.rms(x[(S - 1) - owner * c], O._f(w.final_norm), eps) if rank == owner else \
        torch.zeros(cfg.hidden_size, device=dev)
    dist.broadcast(last, dist.get_global_rank(group, owner) if group is not None else owner, group=group)
    logits = last @ O._f(w.lm_head).t()

    def gather(t):
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous(), group=group)
        return torch.cat(parts)[:S]

    return logits, [gather(k) for k in ks], [gather(v) for v in vs]


def to_blocks(k: torch.Tensor, v: torch.Tensor, block_size: int = 16) -> Tuple[torch.Tensor, torch.Tensor]:
    """[S, Hkv, D] K/V -> the paged layout of ``engine.kv_cache.KVCache``:
    K [nblk, Hkv, 16, D], V [nblk, Hkv, D, 16] (the tail of the last block zero)."""
    S, Hkv, D = k.shape
    nblk = -(-S // block_size)
    kp = k.new_zeros(nblk * block_size, Hkv, D)
    vp = v.new_zeros(nblk * block_size, Hkv, D)
    kp[:S], vp[:S] = k, v
    kb = kp.view(nblk, block_size, Hkv, D).permute(0, 2, 1, 3).contiguous()
    vb = vp.view(nblk, block_size, Hkv, D).permute(0, 2, 3, 1).contiguous()
    return kb, vb
