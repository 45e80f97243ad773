"""Plain PyTorch restatements of every kernel.

They compute in fp32 internally and round at the same points as the fused
kernels (bf16 storage of activations, KV cache and norm outputs), so tests can
compare a kernel with its reference op by op.  On a GPU they are also the
PyTorch + cuBLAS baseline that the native path is measured against.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def linear(x, w, out=None, residual=None, workspace=None, splits=0):
    y = torch.matmul(x.reshape(-1, x.shape[-1]), w.t())
    if residual is not None:
        y = (y.float() + residual.reshape(y.shape).float()).to(y.dtype)
    if out is not None:
        out.view(y.shape).copy_(y)
        return out
    return y


def rmsnorm(x, w, eps, residual=None, out=None):
    if residual is not None:
        residual.copy_((residual.float() + x.float()).to(residual.dtype))
        src = residual
    else:
        src = x
    xf = src.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def inv_freq(rot_dim: int, theta: float, device=None) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float64, device=device) / rot_dim)).float()


def apply_rope(x: torch.Tensor, pos: torch.Tensor, invf: torch.Tensor, rot_dim: int) -> torch.Tensor:
    """Rotate-half RoPE on the first ``rot_dim`` dims of ``x[..., T, H, D]`` (fp32 math)."""
    xf = x.float()
    ang = pos.float()[:, None] * invf[None, :]            # [T, rot/2]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    half = rot_dim // 2
    x1, x2, rest = xf[..., :half], xf[..., half:rot_dim], xf[..., rot_dim:]
    out = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, rest], dim=-1)
    return out.to(x.dtype)


def head_rmsnorm(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def rope_qknorm(qkv, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot_dim, eps):
    T = qkv.shape[0]
    q = qkv[:, : Hq * D].reshape(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].reshape(T, Hkv, D)
    if q_w is not None:
        q = head_rmsnorm(q, q_w, eps)
    if k_w is not None:
        k = head_rmsnorm(k, k_w, eps)
    q = apply_rope(q, positions, invf, rot_dim)
    k = apply_rope(k, positions, invf, rot_dim)
    q_out.view(T, Hq, D).copy_(q)
    if slots is not None:
        bs = k_cache.shape[2]
        valid = slots >= 0
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            # fixed shapes inside a graph: padded rows (slot -1) write into the cache's last block,
            # which the engine keeps out of the allocator as scratch
            scratch = (k_cache.shape[0] - 1) * bs + torch.arange(T, device=slots.device) % bs
            s = torch.where(valid, slots.long(), scratch)
            blk, off = s // bs, s % bs
            k_cache[blk, :, off, :] = k
            v_cache[blk, :, :, off] = v
            return q_out
        s = slots[valid].long()
        blk, off = s // bs, s % bs
        k_cache[blk, :, off, :] = k[valid]
        v_cache[blk, :, :, off] = v[valid]          # V blocks are [Hkv, D, BS]
    return q_out


def gather_kv(cache: torch.Tensor, block_table: torch.Tensor, n: int) -> torch.Tensor:
    """[num_blocks, Hkv, BS, D] + table -> [n, Hkv, D] for one sequence."""
    bs = cache.shape[2]
    nb = (n + bs - 1) // bs
    blocks = cache[block_table[:nb].long()]                # [nb, Hkv, BS, D]
    return blocks.permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[1], cache.shape[3])[:n]


def gather_v(cache: torch.Tensor, block_table: torch.Tensor, n: int) -> torch.Tensor:
    """[num_blocks, Hkv, D, BS] + table -> [n, Hkv, D] for one sequence."""
    bs = cache.shape[3]
    nb = (n + bs - 1) // bs
    blocks = cache[block_table[:nb].long()]                # [nb, Hkv, D, BS]
    return blocks.permute(0, 3, 1, 2).reshape(nb * bs, cache.shape[1], cache.shape[2])[:n]


def attn_decode(q, k_cache, v_cache, block_tables, ctx_lens, out=None, splits=1, workspace=None, scale=None):
    """Decode attention: q [B, Hq, D] against each sequence's paged KV."""
    B, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    G = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lens = ctx_lens.tolist()
    res = torch.empty_like(q) if out is None else out
    for b in range(B):
        n = int(lens[b])
        k = gather_kv(k_cache, block_tables[b], n).float()    # [n, Hkv, D]
        v = gather_v(v_cache, block_tables[b], n).float()
        qb = q[b].float().view(Hkv, G, D)
        s = torch.einsum("hgd,nhd->hgn", qb, k) * scale
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("hgn,nhd->hgd", p, v).reshape(Hq, D)
        res[b].copy_(o.to(q.dtype))
    return res


def attn_decode_batched(q, k_cache, v_cache, block_tables, ctx_lens, out=None, scale=None):
    """Batched form used by the baseline engine: gather -> masked SDPA."""
    B, Hq, D = q.shape
    Hkv, bs = k_cache.shape[1], k_cache.shape[2]
    maxb = block_tables.shape[1]
    k = k_cache[block_tables.long()]                          # [B, maxb, Hkv, BS, D]
    v = v_cache[block_tables.long()]                          # [B, maxb, Hkv, D, BS]
    k = k.permute(0, 2, 1, 3, 4).reshape(B, Hkv, maxb * bs, D)
    v = v.permute(0, 2, 1, 4, 3).reshape(B, Hkv, maxb * bs, D)
    mask = torch.arange(maxb * bs, device=q.device)[None, :] < ctx_lens[:, None]
    o = F.scaled_dot_product_attention(q[:, :, None, :], k, v, attn_mask=mask[:, None, None, :],
                                       scale=scale, enable_gqa=True)
    o = o[:, :, 0, :]
    if out is not None:
        out.copy_(o)
        return out
    return o


def attn_prefill(q, k, v, scale=None, causal=True):
    """q [S, Hq, D], k/v [S, Hkv, D] of one sequence -> [S, Hq, D]."""
    o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
                                       is_causal=causal, scale=scale, enable_gqa=True)
    return o[0].transpose(0, 1)


def moe_route(logits, top_k, renorm) -> Tuple[torch.Tensor, torch.Tensor]:
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, top_k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids.int(), w


def moe_experts(x, ids, wts, w13, w2, num_experts, inter):
    """Reference expert mixture: loop over experts, SwiGLU MLP, weighted sum.
    w13: [E*2I, H] (per expert [gate; up]); w2: [E*H, I]."""
    T, H = x.shape
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    w13 = w13.view(num_experts, 2 * inter, H)
    w2 = w2.view(num_experts, H, inter)
    flat_ids = ids.reshape(-1)
    for e in torch.unique(flat_ids).tolist():
        tok, slot = (ids == e).nonzero(as_tuple=True)
        xe = x[tok]
        gu = torch.matmul(xe, w13[e].t())
        h = (F.silu(gu[:, :inter].float()) * gu[:, inter:].float()).to(x.dtype)
        ye = torch.matmul(h, w2[e].t()).float()
        out.index_add_(0, tok, ye * wts[tok, slot].float()[:, None])
    return out


def swiglu(gu, out=None):
    I = gu.shape[-1] // 2
    y = (F.silu(gu[..., :I].float()) * gu[..., I:].float()).to(gu.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def embed(ids, table, out=None, vocab_start=0):
    local = ids - vocab_start
    ok = (local >= 0) & (local < table.shape[0])
    y = table[local.clamp(0, table.shape[0] - 1)] * ok[:, None].to(table.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def argmax(logits, out=None, out_val=None, index_offset=0):
    v, i = logits.float().max(dim=-1)
    i = i + index_offset
    if out is not None:
        out.copy_(i)
    if out_val is not None:
        out_val.copy_(v)
    return i if out is None else out


def verify_tokens(draft, target, out=None):
    neq = draft != target
    L = draft.shape[1]
    idx = torch.where(neq, torch.arange(L, device=draft.device)[None, :], torch.full_like(draft, L))
    r = idx.min(dim=1).values.int()
    if out is not None:
        out.copy_(r)
        return out
    return r
