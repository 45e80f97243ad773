"""Thin, allocation-explicit wrappers around the sm_100a kernels.

Every function takes its output buffers as arguments (or allocates them once
with the caching allocator when ``out`` is omitted), so the whole decode step
can be captured in a CUDA graph.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import autotune, load_extension


def _C():
    return load_extension()


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
           residual: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
           splits: int = 0, orient: int = -1) -> torch.Tensor:
    """``out = x @ w.T (+ residual)``; tcgen05 GEMM.  ``splits=0`` picks split-K automatically;
    ``orient`` forces the tile orientation (0: activations on the 128-row MMA side, 1: weights)."""
    x2 = x.reshape(-1, x.shape[-1])
    if out is None:
        out = torch.empty(x2.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    if splits == 0 and orient < 0 and autotune._ACTIVE is not None:
        hit = autotune._ACTIVE.get((x2.shape[0], w.shape[0], x2.shape[1]))
        if hit is not None:
            splits, orient = hit
    _C().linear(x2, w, out.view(x2.shape[0], w.shape[0]),
                None if residual is None else residual.reshape(x2.shape[0], w.shape[0]), workspace, splits, orient)
    return out


def linear_cluster(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                   residual: Optional[torch.Tensor] = None, cs: int = 0, wait=None) -> torch.Tensor:
    """``out = x @ w.T (+ residual)`` for decode-sized x (1..128 rows): split-K over a
    thread-block cluster of ``cs`` CTAs (0: automatic) reduced through distributed
    shared memory, one launch and no fp32 workspace.  ``wait = (flags_addr, state,
    nranks)`` (tensor parallelism): x is a gathered buffer and its loads wait until
    every rank's flag reaches ``state[0]``."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    flags, state, nranks = wait if wait is not None else (0, None, 0)
    _C().linear_cluster(x, w, out, residual, cs, flags, state, nranks)
    return out


def swiglu_cluster(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None, cs: int = 0,
                   wait=None) -> torch.Tensor:
    """``silu(x @ gate^T) * (x @ up^T)``, w = [gate; up] ([2I, K], I % 64 == 0), for decode-sized
    x (1..128 rows): one cluster split-K launch whose tiles pair 64 gate rows with the matching
    64 up rows, SwiGLU applied after the DSMEM reduction.  ``wait``: as in :func:`linear_cluster`."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0] // 2, dtype=x.dtype, device=x.device)
    flags, state, nranks = wait if wait is not None else (0, None, 0)
    _C().swiglu_cluster(x, w, out, cs, flags, state, nranks)
    return out


def linear_cluster_w8(x: torch.Tensor, wq: torch.Tensor, scale: torch.Tensor, out: Optional[torch.Tensor] = None,
                      residual: Optional[torch.Tensor] = None, cs: int = 0) -> torch.Tensor:
    """int8 weight-only ``out = (x @ wq.T) * scale (+ residual)`` for decode-sized x: the cluster
    split-K GEMM with each int8 weight tile expanded to bf16 in shared memory."""
    if out is None:
        out = torch.empty(x.shape[0], wq.shape[0], dtype=x.dtype, device=x.device)
    _C().linear_cluster_w8(x, wq, scale, out, residual, cs)
    return out


def qkv_rope_cluster(x, w, q_w, k_w, positions, inv_freq, slots, q_out, k_cache, v_cache, Hq, Hkv, rot_dim, eps,
                     cs: int = 0, wait=None):
    """Packed QKV projection (head_dim 128) with QK-RMSNorm, RoPE and the paged KV
    write in the cluster GEMM's epilogue; same result as ``linear`` + ``rope_qknorm``.
    ``wait``: as in :func:`linear_cluster`."""
    flags, state, nranks = wait if wait is not None else (0, None, 0)
    _C().qkv_rope_cluster(x, w, q_w, k_w, positions, inv_freq, slots, q_out, k_cache, v_cache, Hq, Hkv, rot_dim,
                          eps, cs, flags, state, nranks)
    return q_out


def swiglu_linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                  workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(x @ gate^T) * (x @ up^T), w = [gate; up]; decode shapes (T <= 256) with split-K."""
    T, I = x.shape[0], w.shape[0] // 2
    if out is None:
        out = torch.empty(T, I, dtype=x.dtype, device=x.device)
    if workspace is None:
        workspace = torch.empty(8 * T * 2 * I, dtype=torch.float32, device=x.device)
    _C().swiglu_linear(x, w, out, workspace, 0, None, 0)
    return out


def grouped_linear(xs: torch.Tensor, w: torch.Tensor, offs: torch.Tensor, groups: int, swiglu: bool,
                   max_rows_per_group: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    rows_pg = w.shape[0] // groups
    n_out = rows_pg // 2 if swiglu else rows_pg
    if out is None:
        out = torch.empty(xs.shape[0], n_out, dtype=xs.dtype, device=xs.device)
    _C().grouped_linear(xs, w, offs, out, groups, swiglu, max_rows_per_group)
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    _C().rmsnorm(x, residual, w, out, eps)
    return out


def rope_qknorm(qkv, q_w, k_w, positions, inv_freq, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot_dim, eps):
    _C().rope_qknorm(qkv, q_w, k_w, positions, inv_freq, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot_dim, eps)
    return q_out


def attn_decode(q, k_cache, v_cache, block_tables, ctx_lens, out=None, splits: int = 1, workspace=None,
                scale: Optional[float] = None):
    if out is None:
        out = torch.empty_like(q)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    _C().attn_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, splits, workspace, scale)
    return out


_WORK = {}


def _work_counter(device) -> torch.Tensor:
    """Per-device int32[2] work queue of the decode-attention kernel; zero between
    launches (the kernel's last CTA resets it), so one buffer serves every call."""
    key = torch.device(device).index
    if key not in _WORK:
        _WORK[key] = torch.zeros(2, dtype=torch.int32, device=device)
    return _WORK[key]


def attn_decode_tc(q, k_cache, v_cache, block_tables, ctx_lens, out=None, splits: int = 1, workspace=None,
                   scale: Optional[float] = None, dynamic: bool = True):
    """tcgen05 flash-decode (head_dim 128, group <= 16); same contract as attn_decode.
    Work items (sequence, KV head, chunk of ceil(max_blocks / splits) blocks) are
    handed out dynamically, longest first."""
    if out is None:
        out = torch.empty_like(q)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    work = _work_counter(q.device) if dynamic else torch.empty(0, dtype=torch.int32, device=q.device)
    _C().attn_decode_tc(q, k_cache, v_cache, block_tables, ctx_lens, out, splits, workspace, scale, work)
    return out


def attn_prefill_tc(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, max_q_len: int, out=None,
                    scale: Optional[float] = None, causal: bool = True):
    """tcgen05 flash prefill over the paged cache.  q [T, Hq, D] (D = 64, 128 or 256); causal=False
    lets every query of a sequence see all its keys (bidirectional)."""
    T, Hq, D = q.shape
    if out is None:
        out = torch.empty_like(q)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    _C().attn_prefill_tc(q.view(T, Hq * D), k_cache, v_cache, block_tables, cu_q, ctx_lens, out.view(T, Hq * D),
                         max_q_len, scale, causal)
    return out


def attn_decode_tc_supported(D: int, G: int) -> bool:
    return bool(_C().attn_decode_tc_supported(D, G))


def moe_route(logits, top_k, renorm, ids, wts, counts, offs, cursor):
    _C().moe_route(logits, top_k, renorm, ids, wts, counts, offs, cursor)


def moe_permute(x, ids, offs, cursor, pos, xs):
    _C().moe_permute(x, ids, offs, cursor, pos, xs)


def moe_combine(y, pos, wts, residual, out):
    _C().moe_combine(y, pos, wts, residual, out)
    return out


def embed(ids, table, out=None, vocab_start: int = 0):
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    _C().embed(ids, table, out, vocab_start)
    return out


def swiglu(gu, out=None):
    if out is None:
        out = torch.empty(*gu.shape[:-1], gu.shape[-1] // 2, dtype=gu.dtype, device=gu.device)
    _C().swiglu(gu, out)
    return out


def argmax(logits, out=None, out_val=None, index_offset: int = 0):
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    _C().argmax(logits, out, out_val, index_offset)
    return out


def verify_tokens(draft, target, out=None):
    if out is None:
        out = torch.empty(draft.shape[0], dtype=torch.int32, device=draft.device)
    _C().verify_tokens(draft, target, out)
    return out


def deltanet_decode(mixed, z, ba, conv_w, conv_state, ssm, slots, A_log, dt_bias, norm_w, Hk: int, Hv: int,
                    dk: int, dv: int, eps: float, out=None):
    """Fused gated-DeltaNet decode step (conv, L2 norms, gates, delta rule, gated RMSNorm).
    mixed [B, 2*Hk*dk + Hv*dv] raw projections, z [B, Hv*dv], ba [B, 2*Hv]; states updated in place."""
    if out is None:
        out = torch.empty(mixed.shape[0], Hv * dv, dtype=torch.bfloat16, device=mixed.device)
    _C().deltanet_decode(mixed, z, ba, conv_w, conv_state, ssm, slots, A_log, dt_bias, norm_w, out, Hk, Hv, dk, dv,
                         eps)
    return out


def deltanet_prefill(mixed, z, ba, conv_w, conv_state, ssm, slots, cu, seq_of, A_log, dt_bias, norm_w, Hk: int,
                     Hv: int, dk: int, dv: int, eps: float, out=None, xc=None):
    """Packed multi-sequence gated-DeltaNet prefill (cu: int32 offsets [nseq+1], seq_of: int32 [T])."""
    T = mixed.shape[0]
    if out is None:
        out = torch.empty(T, Hv * dv, dtype=torch.bfloat16, device=mixed.device)
    if xc is None:
        xc = torch.empty(mixed.shape, dtype=torch.float32, device=mixed.device)
    _C().deltanet_prefill(mixed, z, ba, conv_w, conv_state, ssm, slots, cu, seq_of, A_log, dt_bias, norm_w, out, xc,
                          Hk, Hv, dk, dv, eps)
    return out


def linear_w8(x, wq, scale, out=None, residual=None, workspace=None, offs=None, groups: int = 1,
              swiglu: bool = False, max_rows_per_group: int = 0):
    """int8 weight-only GEMM: y = (x @ wq^T) * scale[None, :] (+ residual).  wq int8 [N, K],
    scale f32 [N].  ``offs`` (int32 [groups+1]) = grouped expert mode over ``groups`` weight blocks;
    ``swiglu`` = gate|up weights per group, output silu(gate) * up."""
    rows_pg = wq.shape[0] // (groups if offs is not None else 1)
    n_out = rows_pg // 2 if swiglu else rows_pg
    if out is None:
        out = torch.empty(x.shape[0], n_out, dtype=torch.bfloat16, device=x.device)
    _C().linear_w8(x, wq, scale, out, residual, workspace, offs, groups, swiglu, max_rows_per_group)
    return out


def sample_tokens(logits, temperature, top_k, top_p, seeds, steps, out=None):
    """Fused temperature / top-k / top-p sampling (one CTA per row, no sort); temperature <= 0
    rows are greedy.  temperature, top_p f32 [B]; top_k int32 [B] (0 = off); seeds, steps int64 [B]
    (the Gumbel noise is a hash of (seed, step, token id))."""
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    _C().sample_tokens(logits.contiguous(), temperature, top_k, top_p, seeds, steps, out)
    return out


def patchify(images, size: int, patch: int, merge: int, mean, std, out=None):
    """[B, C, h, w] (f32 / bf16) -> bilinear resize to size x size, (x - mean) / std, patches in
    spatial-merge-group order as bf16 rows [B, (size/patch)^2, C*patch*patch]."""
    B, C = images.shape[:2]
    g = size // patch
    if out is None:
        out = torch.empty(B, g * g, C * patch * patch, dtype=torch.bfloat16, device=images.device)
    _C().patchify(images.contiguous(), size, patch, merge, [float(v) for v in mean], [float(v) for v in std], out)
    return out


def bias_act(y, bias=None, gelu: bool = False):
    """In place: y = act(y + bias), act = tanh-GELU or identity; y bf16 [rows, cols]."""
    _C().bias_act(y, bias, gelu)
    return y


def grouped_linear_wait(xs, w, offs, groups: int, swiglu: bool, max_rows_per_group: int, flags: int, state,
                        nranks: int, epoch_add: int, out=None):
    """grouped_linear whose input rows are written by other GPUs: the TMA producer first waits
    (bounded) until flags[p] >= state[0] + epoch_add for every p < nranks (flags: device address)."""
    rows_pg = w.shape[0] // groups
    n_out = rows_pg // 2 if swiglu else rows_pg
    if out is None:
        out = torch.empty(xs.shape[0], n_out, dtype=xs.dtype, device=xs.device)
    _C().grouped_linear_wait(xs, w, offs, out, groups, swiglu, max_rows_per_group, flags, state, nranks, epoch_add)
    return out


def vit_rope_kv(qkv, pos, N: int, heads: int, D: int, theta: float, q_out, k_cache, v_cache):
    """ViT 2-D RoPE of q and k, q -> q_out, k / v of each image into its own blocks of a paged cache."""
    _C().vit_rope_kv(qkv, pos, N, heads, D, theta, q_out, k_cache, v_cache)
    return q_out
