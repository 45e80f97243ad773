"""Context parallelism for long prefills: ring attention, Ulysses, DeltaNet state passing.

The reference has none of these (its attention materialises S x S scores,
``src/inference_pio/plugins/cpu/c_src/tensor_ops.c:544``, and its DeltaNet runs
token by token, ``:789-808``).  Here a prompt's tokens are split into one
contiguous chunk per rank of a process group:

* ``ring_attention`` -- each rank keeps its query chunk; K/V chunks travel
  around the ring (send to rank+1, receive from rank-1, overlapped with the
  current chunk's math) and partial results are merged with their
  log-sum-exp.  Causal: a KV chunk from a later rank is skipped, the own
  chunk uses the causal mask, earlier chunks attend fully.
* ``ulysses_attention`` -- one all-to-all turns (sequence-sharded, all heads)
  into (full sequence, heads / N), attention runs locally, a second
  all-to-all turns the output back.  Needs query and KV head counts that
  divide by the group size.
* ``deltanet_cp`` -- the gated delta rule's state update is affine in the
  state: over one chunk S_end = P S_0 + Q (P = the chunk run from the
  identity with zero values, Q = the chunk run from zero).  Every rank
  computes its (P, Q), the maps are all-gathered, each rank folds the maps of
  the ranks before it onto the incoming state and then runs its chunk from
  the state it really starts from.

These are the baseline form (torch.distributed point-to-point and
all-to-all, fp32 torch math per chunk), for any backend including gloo.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from ..models.deltanet import chunk_gated_delta_rule


def _group_info(group) -> Tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def attention_with_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                       mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """q [Sq, Hq, D], k/v [Sk, Hkv, D] -> (o [Sq, Hq, D] fp32, lse [Hq, Sq] fp32; -inf where nothing is visible).
    ``mask`` [Sq, Sk] bool, True = visible."""
    Hq, Hkv = q.shape[1], k.shape[1]
    rep = Hq // Hkv
    qf = q.float().transpose(0, 1)                                         # [Hq, Sq, D]
    kf = k.float().transpose(0, 1).repeat_interleave(rep, dim=0)           # [Hq, Sk, D]
    vf = v.float().transpose(0, 1).repeat_interleave(rep, dim=0)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask[None], -math.inf)
    lse = torch.logsumexp(s, dim=-1)                                       # [Hq, Sq]
    p = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[..., None])
    o = (p @ vf).transpose(0, 1)                                           # [Sq, Hq, D]
    return o, lse


def merge_partials(o1, lse1, o2, lse2):
    """Merge two normalised partial attentions over disjoint key sets."""
    m = torch.maximum(lse1, lse2)
    m0 = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w1, w2 = torch.exp(lse1 - m0), torch.exp(lse2 - m0)
    tot = w1 + w2
    lse = torch.where(tot > 0, m0 + torch.log(tot), torch.full_like(m, -math.inf))
    tot = torch.where(tot > 0, tot, torch.ones_like(tot))
    a1 = (w1 / tot).transpose(0, 1)[..., None]
    a2 = (w2 / tot).transpose(0, 1)[..., None]
    return o1 * a1 + o2 * a2, lse


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                   scale: Optional[float] = None, group=None) -> torch.Tensor:
    """This rank's query chunk attends over every rank's K/V chunk (chunks are
    contiguous, rank order = sequence order, equal lengths)."""
    rank, world = _group_info(group)
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    S = q.shape[0]
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    kv = torch.stack([k, v]).contiguous()
    o = torch.zeros(S, q.shape[1], q.shape[2], dtype=torch.float32, device=q.device)
    lse = torch.full((q.shape[1], S), -math.inf, dtype=torch.float32, device=q.device)
    own_mask = torch.ones(S, S, dtype=torch.bool, device=q.device).tril() if causal else None
    for step in range(world):
        src = (rank - step) % world
        reqs = []
        if step + 1 < world:  # pass the chunk on while this one is used
            recv = torch.empty_like(kv)
            reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, kv, nxt, group),
                                           dist.P2POp(dist.irecv, recv, prv, group)])
        if not (causal and src > rank):
            oi, li = attention_with_lse(q, kv[0], kv[1], scale, own_mask if (causal and src == rank) else None)
            o, lse = merge_partials(o, lse, oi, li)
        for r in reqs:
            r.wait()
        if step + 1 < world:
            kv = recv
    return o.to(q.dtype)


def _a2a(x: torch.Tensor, group) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)  # contiguous (empty_like would keep x's strides)
    dist.all_to_all_single(out, x, group=group)
    return out


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                      scale: Optional[float] = None, group=None) -> torch.Tensor:
    """q [S/N, Hq, D], k/v [S/N, Hkv, D] (this rank's sequence chunk) -> [S/N, Hq, D]."""
    rank, world = _group_info(group)
    Sl, Hq, D = q.shape
    Hkv = k.shape[1]
    if Hq % world or Hkv % world:
        raise ValueError(f"ulysses: {Hq} query / {Hkv} KV heads do not divide by {world} ranks")

    def seq_to_heads(x):  # [Sl, H, D] -> [world*Sl, H/world, D]: send head group j to rank j
        H = x.shape[1]
        x = x.reshape(Sl, world, H // world, D).transpose(0, 1)          # [world, Sl, H/w, D]
        return _a2a(x, group).reshape(world * Sl, H // world, D)        # received: [src rank, Sl, H/w, D]

    qh, kh, vh = seq_to_heads(q), seq_to_heads(k), seq_to_heads(v)
    mask = torch.ones(world * Sl, world * Sl, dtype=torch.bool, device=q.device).tril() if causal else None
    o, _ = attention_with_lse(qh, kh, vh, scale if scale is not None else D ** -0.5, mask)
    o = o.to(q.dtype).reshape(world, Sl, Hq // world, D)                 # [seq chunk j, Sl, my heads, D]
    back = _a2a(o, group)                                                # [head group j, Sl, H/w, D]
    return back.transpose(0, 1).reshape(Sl, Hq, D)


def deltanet_cp(q, k, v, g, beta, state: Optional[torch.Tensor] = None, chunk: int = 64, group=None):
    """Gated delta rule over a sequence split into contiguous per-rank chunks.

    q, k: [H, L_local, dk]; v: [H, L_local, dv]; g, beta: [H, L_local]; ``state`` [H, dk, dv] is the
    state before the first token of rank 0's chunk (zeros if None; the same on every rank).
    Returns (o [H, L_local, dv], final state after the LAST rank's chunk, identical on every rank)."""
    rank, world = _group_info(group)
    H, _, dk = q.shape
    dv = v.shape[-1]
    f32 = dict(dtype=torch.float32, device=q.device)
    if state is None:
        state = torch.zeros(H, dk, dv, **f32)
    eye = torch.eye(dk, **f32).expand(H, dk, dk).contiguous()
    _, P = chunk_gated_delta_rule(q, k, torch.zeros(H, k.shape[1], dk, **f32), g, beta, eye, chunk)
    _, Q = chunk_gated_delta_rule(q, k, v, g, beta, torch.zeros(H, dk, dv, **f32), chunk)
    Ps = [torch.empty_like(P) for _ in range(world)]
    Qs = [torch.empty_like(Q) for _ in range(world)]
    dist.all_gather(Ps, P.contiguous(), group=group)
    dist.all_gather(Qs, Q.contiguous(), group=group)
    S = state.float()
    for j in range(rank):
        S = Ps[j] @ S + Qs[j]
    o, S_mine = chunk_gated_delta_rule(q, k, v, g, beta, S, chunk)
    S_end = S_mine
    for j in range(rank + 1, world):
        S_end = Ps[j] @ S_end + Qs[j]
    return o, S_end
