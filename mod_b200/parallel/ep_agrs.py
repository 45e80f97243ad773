"""Expert parallelism as all-gather -> local experts -> reduce-scatter over NVLink
multicast, for decode-sized steps (``csrc/cuda/ep_agrs.cu``).

Every rank multicasts its tokens' normed rows and routing choices to every rank
(one store per 16 bytes, replicated by the switch), runs its local experts on
every token that picked one, and each token's owner reads the sum of the ranks'
weighted expert outputs with one ``multimem.ld_reduce``, fused with the
residual add and the next RMSNorm.  Two cross-rank waits per MoE layer and no
count exchange: every rank sees every token's expert ids, so the placement of
the local rows is computed locally (deterministically).

Steps larger than the decode capacity (prefill), non-deferred calls and MoE
blocks with a shared expert go to the point-to-point dispatch/combine
(:class:`mod_b200.parallel.ep.FusedEPMoE`).

The reference's MoE block loops over experts on one device
(``pio/models/qwen3_coder_30b/model.py:308-353``).
"""
from __future__ import annotations

from typing import Dict

import torch
import torch.distributed as dist


def agrs_layout(world: int, cap: int, K: int, H: int) -> Dict[str, int]:
    """Byte offsets of the symmetric buffer, each region on a 256-byte boundary:
    ``gx`` [N*cap, H] bf16, ``gid`` / ``gw`` [N*cap, K] int32 / fp32, ``gcnt`` [N] u32,
    ``part`` [N*cap, H] bf16, ``ag_flag`` / ``rs_flag`` [N] u32."""
    al = lambda x: (x + 255) // 256 * 256  # noqa: E731
    rows = world * cap
    L = {"gx": 0}
    L["gid"] = al(rows * H * 2)
    L["gw"] = al(L["gid"] + rows * K * 4)
    L["gcnt"] = al(L["gw"] + rows * K * 4)
    L["part"] = al(L["gcnt"] + world * 4)
    L["ag_flag"] = al(L["part"] + rows * H * 2)
    L["rs_flag"] = al(L["ag_flag"] + world * 4)
    L["total"] = al(L["rs_flag"] + world * 4)
    return L


def place_reference(ids, counts, rank: int, El: int, cap: int):
    """The placement ``ep_agrs_place_kernel`` computes, as plain Python: the pairs
    (rank r, token t < counts[r], k) whose expert is local, ordered by local expert
    and then by (r, t, k).  Returns ``offs`` [El + 1] and ``slot`` {(g, k): row},
    g = r * cap + t.  ``ids`` is indexable as ids[g][k] (global expert ids)."""
    pairs = []
    for r, c in enumerate(counts):
        for t in range(c):
            g = r * cap + t
            for k, e in enumerate(ids[g]):
                le = int(e) - rank * El
                if 0 <= le < El:
                    pairs.append((le, g, k))
    pairs.sort(key=lambda p: p[0])  # stable: keeps (r, t, k) order within an expert
    offs = [0] * (El + 1)
    for le, _, _ in pairs:
        offs[le + 1] += 1
    for e in range(El):
        offs[e + 1] += offs[e]
    return offs, {(g, k): i for i, (_, g, k) in enumerate(pairs)}


class AgRsEPMoE:
    """Callable ``(x [T, H] normed rows, moe_weights, defer) ->`` a pending
    combine (``add_norm(residual, w, eps)``), or the fallback's result."""

    def __init__(self, cfg, backend, max_tokens: int, fallback, group=None):
        from ..ops import load_extension, native
        from .symm import SymmetricBuffer

        self.C, self.N = load_extension(), native
        self.cfg, self.be, self.fallback, self.group = cfg, backend, fallback, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        E, self.K, self.H = cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size
        assert E % self.world == 0
        self.El = E // self.world
        self.cap = max(1, int(max_tokens))
        self.supports_defer = True
        L = agrs_layout(self.world, self.cap, self.K, self.H)
        self.L = L
        self.buf = SymmetricBuffer(L["total"], group)
        self.own, self.mc = self.buf.own, self.buf.mc
        self.offsets = torch.tensor([L["gx"], L["gid"], L["gw"], L["gcnt"], L["part"], L["ag_flag"]],
                                    dtype=torch.int64)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.state = torch.zeros(8, dtype=torch.int32, device=dev)
        self.max_pairs = self.world * self.cap * self.K
        self.xs = torch.empty(self.max_pairs, self.H, dtype=torch.bfloat16, device=dev)
        self.slot_of = torch.empty(self.max_pairs, dtype=torch.int32, device=dev)
        self.offs = torch.zeros(self.El + 1, dtype=torch.int32, device=dev)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.place_grid = max(1, min(sms, -(-self.max_pairs // 32)))

    def covers(self, mo) -> bool:
        E = self.El * self.world
        return (mo.shared is None and E <= 512 and self.H % 256 == 0
                and mo.router.dtype == torch.bfloat16 and isinstance(mo.w13, torch.Tensor))

    def __call__(self, x: torch.Tensor, mo, defer: bool = False):
        T = x.shape[0]
        if torch.cuda.is_current_stream_capturing():
            use = defer and self.covers(mo) and T <= self.cap
        else:  # every rank must take the same path
            flag = torch.tensor([T if (defer and self.covers(mo)) else 1 << 30], dtype=torch.int64,
                                device=x.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
            use = int(flag.item()) <= self.cap
        if not use:
            return self.fallback(x, mo, defer=defer)
        C, N = self.C, self.N
        x = x.contiguous()
        args = (self.own, self.mc, self.rank, self.world, self.cap, self.K, self.El)
        logits = self.be.linear(x, mo.router) if T > 0 else x.new_empty(0, self.El * self.world)
        C.ep_agrs_publish(*args, self.offsets, self.state, x, logits, bool(self.cfg.norm_topk_prob))
        C.ep_agrs_place(*args, self.H, self.offsets, self.state, self.xs, self.slot_of, self.offs, self.place_grid)
        per_expert = max(1, (self.world * max(T, 1) * self.K) // (self.El * self.world))
        mr = min(self.max_pairs, 4 * per_expert)
        h = N.grouped_linear(self.xs, mo.w13, self.offs, self.El, True, mr)
        y = N.grouped_linear(h, mo.w2, self.offs, self.El, False, mr)
        C.ep_agrs_combine(*args, self.H, self.offsets, self.state, self.slot_of, y)
        return AgRsPending(self, T)


class AgRsPending:
    """This rank's weighted expert sums are in its ``part`` rows; ``add_norm``
    reduces every rank's rows of this rank's tokens in the switch, adds them to
    the residual and returns the next RMSNorm, in one kernel."""

    def __init__(self, moe: AgRsEPMoE, T: int):
        self.moe, self.T = moe, T

    def add_norm(self, residual: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        m = self.moe
        out = torch.empty_like(residual)
        m.C.tp_nvls_reduce(m.own, m.mc, m.rank, m.world, True, residual.shape[0], m.cap, False, m.H, m.L["gx"],
                           m.L["part"], m.L["ag_flag"], m.L["rs_flag"], m.state, None, residual, w, eps, out)
        return out
