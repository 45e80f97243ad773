"""Expert parallelism for MoE layers.

Layout: every rank serves its own batch slice with a full (replicated) copy
of attention and router weights ("DP attention") and owns experts
``[rank*El, (rank+1)*El)`` with ``El = E / world``.

* :class:`FusedEPMoE` - the product path.  Dispatch and combine are CUDA
  kernels that move token rows over NVLink with peer stores into IPC-mapped
  exchange buffers (``csrc/cuda/ep.cu``); the expert math is the tcgen05
  grouped GEMM.  No NCCL call, no host synchronisation, CUDA-graph safe.
* :class:`NcclEPMoE` - the baseline: routing on the device, then
  ``all_to_all_single`` (NCCL, or gloo on CPU) with host-side split sizes, the
  experts as per-expert ``torch.matmul`` (cuBLAS), and a second all-to-all back.

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
        self.small = _EpContext(self.C, self.world, self.rank, self.El, K, self.H, max_tokens, group)
        self.large = (_EpContext(self.C, self.world, self.rank, self.El, K, self.H, prefill_tokens, group)
                      if prefill_tokens > max_tokens else self.small)

    def _chunk(self, ctx, x, mo):
        cfg, N = self.cfg, self.N
        T = x.shape[0]
        dev = x.device
        E = cfg.num_experts
        logits = self.be.linear(x, mo.router)
        ids = torch.empty(T, self.K, dtype=torch.int32, device=dev)
        wts = torch.empty(T, self.K, dtype=torch.float32, device=dev)
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        offs_g = torch.empty(E + 1, dtype=torch.int32, device=dev)
        cursor = torch.empty(E, dtype=torch.int32, device=dev)
        N.moe_route(logits, self.K, cfg.norm_topk_prob, ids, wts, counts, offs_g, cursor)
        emap = torch.empty(T * self.K, dtype=torch.int32, device=dev)
        # one kernel: counts all-gather, then every row stored at its expert-ordered position in
        # the owner's receive region; the gate/up GEMM waits for the senders' flags itself
        self.C.ep_dispatch2(ctx.buf.peers, ctx.state, self.rank, ctx.cap, self.El, x, ids, counts, offs_g, cursor,
                            emap, ctx.offs)
        rows = ctx.xs_direct.shape[0]
        exp_rows = max(1, (self.world * T * self.K) // max(1, self.El * self.world))
        mr = min(rows, 4 * exp_rows)
        h = N.grouped_linear_wait(ctx.xs_direct, mo.w13, ctx.offs, self.El, True, mr, ctx.flag_addr, ctx.state,
                                  self.world, 1)
        # (returning rows from the down GEMM's epilogue measured slower: its per-element 2-byte
        # peer stores make 64-byte NVLink writes, where the copy kernel writes 512 bytes per warp)
        y = N.grouped_linear(h, mo.w2, ctx.offs, self.El, False, mr)
        out = torch.empty_like(x)
        self.C.ep_combine2(ctx.buf.peers, ctx.state, self.rank, ctx.cap, self.El, ctx.offs, y, emap, wts, None, out)
        return out

    def __call__(self, x: torch.Tensor, mo) -> torch.Tensor:
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
        outs = []
        for c in range(n):
            xc = x[c * ctx.max_tokens:(c + 1) * ctx.max_tokens]
            outs.append(self._chunk(ctx, xc.contiguous(), mo))
        out = torch.cat(outs, 0) if len(outs) > 1 else outs[0]
        if mo.shared is not None:
            sh = self.be.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down).float()
            out = (out.float() + torch.sigmoid(x.float() @ mo.shared_gate.float().t()) * sh).to(x.dtype)
        return out


class NcclEPMoE:
    """Baseline EP MoE: device routing, NCCL/gloo all-to-all, per-expert matmuls."""

    def __init__(self, cfg, backend, group=None):
        self.cfg, self.be, self.group = cfg, backend, group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.El = cfg.num_experts // self.world
        self.K = cfg.num_experts_per_tok

    def __call__(self, x: torch.Tensor, mo) -> torch.Tensor:
        cfg, W, El, K = self.cfg, self.world, self.El, self.K
        T, H = x.shape
        logits = R.linear(x, mo.router)
        ids, wts = R.moe_route(logits, K, cfg.norm_topk_prob)
        flat = ids.reshape(-1).long()
        dst = flat // El
        order = torch.argsort(dst, stable=True)
        send_counts = torch.bincount(dst, minlength=W)
        send_x = x[order // K]
        send_e = (flat[order] % El).to(torch.int32)
        sc = send_counts.tolist()
        if W > 1:
            rc_t = torch.empty_like(send_counts)
            dist.all_to_all_single(rc_t, send_counts, group=self.group)
            rc = rc_t.tolist()
            recv_x = x.new_empty(sum(rc), H)
            recv_e = send_e.new_empty(sum(rc))
            dist.all_to_all_single(recv_x, send_x, rc, sc, group=self.group)
            dist.all_to_all_single(recv_e, send_e, rc, sc, group=self.group)
        else:
            rc, recv_x, recv_e = sc, send_x, send_e
        y = torch.zeros_like(recv_x)
        I = cfg.moe_intermediate_size
        w13 = mo.w13.view(El, 2 * I, H)
        w2 = mo.w2.view(El, H, I)
        for e in torch.unique(recv_e).tolist():
            m = recv_e == e
            gu = R.linear(recv_x[m], w13[e])
            y[m] = R.linear(R.swiglu(gu), w2[e])
        if W > 1:
            back = torch.empty_like(send_x)
            dist.all_to_all_single(back, y, sc, rc, group=self.group)
        else:
            back = y
        out_pairs = torch.empty_like(back)
        out_pairs[order] = back
        out = (out_pairs.view(T, K, H).float() * wts[..., None]).sum(1)
        if mo.shared is not None:
            sh = self.be.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down).float()
            out = out + torch.sigmoid(x.float() @ mo.shared_gate.float().t()) * sh
        return out.to(x.dtype)
