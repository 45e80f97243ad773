"""Expert parallelism for MoE layers.

Layout: every rank serves its own batch slice with a full (replicated) copy
of attention and router weights ("DP attention") and owns experts
``[rank*El, (rank+1)*El)`` with ``El = E / world``.

* :class:`FusedEPMoE` - the product path.  Dispatch and combine are CUDA
  kernels that move token rows over NVLink with peer stores into IPC-mapped
  exchange buffers (``csrc/cuda/ep.cu``); the expert math is the tcgen05
  grouped GEMM.  No NCCL call, no host synchronisation, CUDA-graph safe.
* :class:`NcclEPMoE` - the baseline: routing on the device, fixed-capacity
  ``all_to_all_single`` (NCCL, or gloo on CPU), the experts as two grouped
  library GEMMs with device-side offsets, and a second all-to-all back; no
  host synchronisation, so it is CUDA-graph capturable.

Both return ``sum_k w[t,k] * expert_k(x[t])`` for the local tokens (the
residual is added by the next fused add + RMSNorm).  The reference has no
expert parallelism (``pio/models/qwen3_coder_30b/model.py:291-353``).
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops import reference as R


class ExchangeBuffer:
    """One cudaMalloc'd buffer per rank, mapped into every peer with CUDA IPC.
    ``peers`` is a device int64 tensor of every rank's base address in this
    process's address space (own rank included)."""

    def __init__(self, nbytes: int, group=None):
        from ..ops import load_extension

        C = load_extension()
        self.C = C
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.ptr, handle = C.ipc_alloc(int(nbytes))
        if self.world > 1:
            handles: List[bytes] = [None] * self.world  # type: ignore
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        addrs = []
        self.opened = []
        for r, h in enumerate(handles):
            if r == self.rank:
                addrs.append(self.ptr)
            else:
                p = C.ipc_open(h)
                self.opened.append(p)
                addrs.append(p)
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=torch.cuda.current_device())
        if self.world > 1:
            dist.barrier(group=group)

    def close(self) -> None:
        for p in self.opened:
            self.C.ipc_close(p)
        self.opened = []
        if self.ptr:
            self.C.ipc_free(self.ptr)
            self.ptr = 0


class _EpContext:
    """Exchange buffer + device state for one capacity (max tokens per call)."""

    def __init__(self, C, world, rank, El, K, H, max_tokens, group):
        self.max_tokens = max_tokens
        self.cap = max_tokens * K
        self.buf = ExchangeBuffer(C.ep_buffer_bytes(world, self.cap, H), group)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.state = torch.zeros(8 + world, dtype=torch.int32, device=dev)
        E = El * world
        # fused route + dispatch: counts / cursor / barrier counters (kept zero between calls), fp32 logits
        self.route_scratch = torch.zeros(2 * E + 2, dtype=torch.int32, device=dev)
        self.logits = torch.empty(max_tokens * E, dtype=torch.float32, device=dev)
        rows = world * self.cap
        self.row_pos = torch.empty(rows, dtype=torch.int32, device=dev)
        self.offs = torch.zeros(El + 1, dtype=torch.int32, device=dev)
        self.xs = torch.empty(rows, H, dtype=torch.bfloat16, device=dev)
        self.abort = torch.zeros(1, dtype=torch.int32, device=dev)
        # direct placement: senders write rows into this rank's receive region in expert order
        self.xs_direct = C.wrap_bf16(C.ep_recv_addr(self.buf.peers, rank, self.cap, H), rows, H)
        self.flag_addr = C.ep_flag_addr(self.buf.peers, rank, self.cap, H)


class FusedEPMoE:
    """Callable ``(x [T, H], moe_weights) -> [T, H]`` for one EP rank.

    Two exchange contexts: a small one sized for a decode step (the one used
    inside CUDA graphs) and a large one for prefill, which is processed in
    chunks; all ranks run the same number of rounds."""

    def __init__(self, cfg, backend, max_tokens: int, group=None, prefill_tokens: int = 1024):
        from ..ops import load_extension, native

        self.C = load_extension()
        self.N = native
        self.cfg, self.be = cfg, backend
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.group = group
        E, K = cfg.num_experts, cfg.num_experts_per_tok
        assert E % self.world == 0, "experts must divide evenly across ranks"
        self.El = E // self.world
        self.K = K
        self.H = cfg.hidden_size
        import os

        # MB_EP_FUSED_ROUTE=0 keeps the separate router GEMM / top-k / dispatch launches (A/B timing)
        self.fused_route = self.H % 256 == 0 and os.environ.get("MB_EP_FUSED_ROUTE", "1") != "0"
        # the decoder may leave the combine's weighted sum to the next add + RMSNorm (MB_EP_DEFER=0: off)
        self.supports_defer = os.environ.get("MB_EP_DEFER", "1") != "0"
        # MB_EP_TRACE=1: the route + dispatch kernel records %globaltimer at its phase boundaries here
        self.trace = (torch.zeros(8, dtype=torch.int64, device=torch.device("cuda", torch.cuda.current_device()))
                      if os.environ.get("MB_EP_TRACE") == "1" else None)
        self.small = _EpContext(self.C, self.world, self.rank, self.El, K, self.H, max_tokens, group)
        self.large = (_EpContext(self.C, self.world, self.rank, self.El, K, self.H, prefill_tokens, group)
                      if prefill_tokens > max_tokens else self.small)

    def _chunk(self, ctx, x, mo, defer=False):
        cfg, N = self.cfg, self.N
        T = x.shape[0]
        dev = x.device
        E = cfg.num_experts
        ids = torch.empty(T, self.K, dtype=torch.int32, device=dev)
        wts = torch.empty(T, self.K, dtype=torch.float32, device=dev)
        emap = torch.empty(T * self.K, dtype=torch.int32, device=dev)
        # single rank with a deferred combine: the weighted sum reads the expert rows where the down GEMM
        # wrote them (row of each pair in the expert-ordered buffer), so no rows are sent back
        local = defer and self.world == 1 and self.fused_route
        pmap = torch.empty(T * self.K, dtype=torch.int32, device=dev) if local else None
        if self.fused_route:
            # one kernel: router GEMV, top-k, counts exchange, and every row stored at its
            # expert-ordered position in the owner's receive region
            self.C.ep_route_dispatch(ctx.buf.peers, ctx.state, self.rank, ctx.cap, self.El, x, mo.router, self.K,
                                     cfg.norm_topk_prob, ids, wts, emap, ctx.offs, ctx.route_scratch, ctx.logits,
                                     pmap, self.trace)
        else:
            logits = self.be.linear(x, mo.router)
            counts = torch.empty(E, dtype=torch.int32, device=dev)
            offs_g = torch.empty(E + 1, dtype=torch.int32, device=dev)
            cursor = torch.empty(E, dtype=torch.int32, device=dev)
            N.moe_route(logits, self.K, cfg.norm_topk_prob, ids, wts, counts, offs_g, cursor)
            # counts all-gather, then every row stored at its expert-ordered position in the
            # owner's receive region; the gate/up GEMM waits for the senders' flags itself
            self.C.ep_dispatch2(ctx.buf.peers, ctx.state, self.rank, ctx.cap, self.El, x, ids, counts, offs_g,
                                cursor, emap, ctx.offs)
        rows = ctx.xs_direct.shape[0]
        exp_rows = max(1, (self.world * T * self.K) // max(1, self.El * self.world))
        mr = min(rows, 4 * exp_rows)
        h = N.grouped_linear_wait(ctx.xs_direct, mo.w13, ctx.offs, self.El, True, mr, ctx.flag_addr, ctx.state,
                                  self.world, 1)
        # (returning rows from the down GEMM's epilogue measured slower: its per-element 2-byte
        # peer stores make 64-byte NVLink writes, where the copy kernel writes 512 bytes per warp)
        y = N.grouped_linear(h, mo.w2, ctx.offs, self.El, False, mr)
        if local:
            return PendingCombine(self, ctx, pmap, wts, T, rows=y)
        if defer:
            # rows go back now; the weighted sum happens inside the next add + RMSNorm
            self.C.ep_combine_send(ctx.buf.peers, ctx.state, self.rank, ctx.cap, self.El, ctx.offs, y, self.H)
            return PendingCombine(self, ctx, emap, wts, T)
        out = torch.empty_like(x)
        self.C.ep_combine2(ctx.buf.peers, ctx.state, self.rank, ctx.cap, self.El, ctx.offs, y, emap, wts, None, out)
        return out

    def __call__(self, x: torch.Tensor, mo, defer: bool = False):
        """``defer=True`` (single exchange round, no shared expert): returns a
        :class:`PendingCombine` whose ``add_norm`` finishes the combine inside
        the next residual add + RMSNorm, one kernel instead of two."""
        T = x.shape[0]
        if torch.cuda.is_current_stream_capturing():
            assert T <= self.small.max_tokens, "captured EP step exceeds the decode exchange capacity"
            ctx, n = self.small, 1
        else:
            tmax = T
            if self.world > 1:  # all ranks must pick the same context and round count
                t = torch.tensor([T], dtype=torch.int64, device=x.device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
                tmax = int(t.item())
            ctx = self.small if tmax <= self.small.max_tokens else self.large
            n = max(1, -(-tmax // ctx.max_tokens))
        if defer and n == 1 and mo.shared is None and self.H in (256, 512, 1024, 2048, 3072, 4096):
            return self._chunk(ctx, x.contiguous(), mo, defer=True)
        outs = []
        for c in range(n):
            xc = x[c * ctx.max_tokens:(c + 1) * ctx.max_tokens]
            outs.append(self._chunk(ctx, xc.contiguous(), mo))
        out = torch.cat(outs, 0) if len(outs) > 1 else outs[0]
        if mo.shared is not None:
            sh = self.be.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down).float()
            out = (out.float() + torch.sigmoid(x.float() @ mo.shared_gate.float().t()) * sh).to(x.dtype)
        return out


class PendingCombine:
    """An EP MoE output whose expert rows have been returned to this rank but
    not yet summed.  ``add_norm(residual, w, eps)`` does, in one kernel,
    residual += sum_k w_k * row_k and returns rmsnorm(residual) * w."""

    def __init__(self, moe, ctx, emap, wts, T, rows=None):
        self.moe, self.ctx, self.emap, self.wts, self.T = moe, ctx, emap, wts, T
        self.rows = rows  # single rank: expert output rows read in place (emap indexes them)

    def add_norm(self, residual: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        m, ctx = self.moe, self.ctx
        out = torch.empty_like(residual)
        m.C.ep_combine_norm(ctx.buf.peers, ctx.state, m.rank, ctx.cap, m.El, self.emap, self.wts, residual, w, out,
                            eps, self.rows)
        return out


def _grouped_mm_available(device) -> bool:
    """Whether torch's grouped GEMM (a library kernel with device-side group
    offsets) runs on this device; probed once per process."""
    global _GMM_OK
    if _GMM_OK is None:
        _GMM_OK = False
        if device.type == "cuda" and hasattr(torch, "_grouped_mm"):
            try:
                a = torch.randn(32, 64, device=device, dtype=torch.bfloat16)
                b = torch.randn(2, 128, 64, device=device, dtype=torch.bfloat16).transpose(1, 2)
                offs = torch.tensor([16, 32], dtype=torch.int32, device=device)
                y = torch._grouped_mm(a, b, offs=offs)
                ref = torch.cat([a[:16] @ b[0], a[16:] @ b[1]])
                _GMM_OK = bool(torch.allclose(y.float(), ref.float(), rtol=2e-2, atol=2e-1))
            except Exception:
                _GMM_OK = False
    return _GMM_OK


_GMM_OK = None


class NcclEPMoE:
    """Baseline EP MoE built only from library calls: cuBLAS router GEMM, torch
    top-k, NCCL ``all_to_all_single`` and torch's grouped GEMM for the experts.

    It is written to be a fair comparator, not a strawman: no host
    synchronisation and fixed shapes, so a decode step is CUDA-graph
    capturable.  Every rank sends a fixed-capacity block of ``T*K`` rows to
    every peer (slot ``dst*cap + i`` for the i-th pair routed to ``dst``;
    unused slots carry expert id -1), the owner sorts the received rows by
    local expert on the device, runs gate/up + SwiGLU + down as two grouped
    GEMMs with device-side offsets, scatters the rows back to their slots and
    a second all-to-all returns them; the source sums ``w * y`` over its k
    slots.  Prefill is processed in chunks of ``chunk`` tokens so the
    fixed-capacity buffers stay small; all ranks run the same chunk count.
    Where the grouped GEMM is unavailable (CPU) the experts run one
    ``torch.matmul`` pair per expert.

    The reference's MoE block loops over experts with a host sync per top-k
    slot (``pio/models/qwen3_coder_30b/model.py:308-353``)."""

    def __init__(self, cfg, backend, group=None, chunk: int = 256, max_tokens: int = 256):
        self.cfg, self.be, self.group = cfg, backend, group
        self.max_tokens = max_tokens  # tokens per call inside a captured step (the same on every rank)
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.El = cfg.num_experts // self.world
        self.K = cfg.num_experts_per_tok
        self.chunk = chunk

    def _experts(self, xs, key, counts, mo):
        """xs rows sorted by local expert (padding rows, key == El, last)."""
        cfg, El = self.cfg, self.El
        I, H = cfg.moe_intermediate_size, cfg.hidden_size
        w13 = mo.w13.view(El, 2 * I, H)
        w2 = mo.w2.view(El, H, I)
        if _grouped_mm_available(xs.device):
            offs = torch.cumsum(counts[:El], 0, dtype=torch.int32)
            gu = torch._grouped_mm(xs, w13.transpose(1, 2), offs=offs)
            h = R.swiglu(gu)
            y = torch._grouped_mm(h, w2.transpose(1, 2), offs=offs)
            valid = torch.arange(xs.shape[0], device=xs.device) < offs[-1]
            return y * valid[:, None].to(y.dtype)
        y = torch.zeros_like(xs)
        ends = torch.cumsum(counts, 0).tolist()
        start = 0
        for e in range(El):
            end = ends[e]
            if end > start:
                y[start:end] = R.linear(R.swiglu(R.linear(xs[start:end], w13[e])), w2[e])
            start = end
        return y

    def _call(self, x: torch.Tensor, mo, tcap: int) -> torch.Tensor:
        cfg, W, El, K = self.cfg, self.world, self.El, self.K
        T, H = x.shape
        dev = x.device
        logits = R.linear(x, mo.router)
        ids, wts = R.moe_route(logits, K, cfg.norm_topk_prob)
        flat = ids.reshape(-1).long()                                  # [T*K] global expert ids
        dst = flat // El
        cap = tcap * K                           # rows per (source, owner) block, equal on every rank
        onehot = F.one_hot(dst, W)                                     # [TK, W]
        idx = (onehot.cumsum(0) - 1).gather(1, dst[:, None]).squeeze(1)
        slot = dst * cap + idx                                         # row of each pair in the send buffer
        send_x = x.new_zeros(W * cap, H)
        send_x.index_copy_(0, slot, x.repeat_interleave(K, dim=0))
        send_e = torch.full((W * cap,), -1, dtype=torch.int32, device=dev)
        send_e.index_copy_(0, slot, (flat % El).to(torch.int32))
        if W > 1:
            recv_x = torch.empty_like(send_x)
            recv_e = torch.empty_like(send_e)
            dist.all_to_all_single(recv_e, send_e, group=self.group)
            dist.all_to_all_single(recv_x, send_x, group=self.group)
        else:
            recv_x, recv_e = send_x, send_e
        key = torch.where(recv_e >= 0, recv_e, torch.full_like(recv_e, El)).long()
        order = torch.argsort(key, stable=True)
        counts = torch.zeros(El + 1, dtype=torch.int64, device=dev).scatter_add_(0, key, torch.ones_like(key))
        ys = self._experts(recv_x.index_select(0, order), key, counts, mo)
        y_recv = torch.empty_like(ys).index_copy_(0, order, ys)
        if W > 1:
            back = torch.empty_like(y_recv)
            dist.all_to_all_single(back, y_recv, group=self.group)
        else:
            back = y_recv
        pairs = back.index_select(0, slot).view(T, K, H).float()
        out = (pairs * wts[..., None].float()).sum(1)
        if mo.shared is not None:
            sh = self.be.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down).float()
            out = out + torch.sigmoid(x.float() @ mo.shared_gate.float().t()) * sh
        return out.to(x.dtype)

    def __call__(self, x: torch.Tensor, mo) -> torch.Tensor:
        T = x.shape[0]
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            assert T <= self.max_tokens, "captured baseline EP step exceeds max_tokens"
            return self._call(x, mo, self.max_tokens)
        tmax = T
        if self.world > 1:  # every rank runs the same number of exchanges
            t = torch.tensor([T], dtype=torch.int64, device=x.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            tmax = int(t.item())
        n = max(1, -(-tmax // self.chunk))
        tcap = min(tmax, self.chunk)
        outs = [self._call(x[c * self.chunk:(c + 1) * self.chunk].contiguous(), mo, tcap) for c in range(n)]
        return torch.cat(outs, 0) if n > 1 else outs[0]
