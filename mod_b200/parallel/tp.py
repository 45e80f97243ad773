"""Tensor parallelism with sequence-parallel residual stream.

Rank r owns token rows [r*pr, (r+1)*pr) of the residual stream (pr = padded
tokens / ranks).  Each layer boundary is

    all-gather(normed shard) -> column-parallel GEMM      (QKV, gate/up)
    row-parallel GEMM -> reduce-scatter (+ residual, + next RMSNorm)   (o_proj, down)

:class:`FusedTP` does both boundaries with the kernels in ``csrc/cuda/gemm.cu``
and ``csrc/cuda/tp.cu``: the fused reduce kernel that produces a rank's
normed shard stores it straight into every rank's gathered buffer over NVLink
(each byte crosses once) and releases a flag; the next GEMM waits on those
flags inside its TMA producer and reads locally.  The row-parallel GEMM stores
each partial row once into its owner's slot (from the epilogue, or after a
split-K reduction); the owner's reduce kernel sums the slots in rank order,
adds the residual, applies the next RMSNorm and pushes the new shard.  :class:`NcclTP` is the baseline: NCCL all-gather /
reduce-scatter around cuBLAS GEMMs.

The reference has tensor-parallel settings only as configuration strings
(``pio/models/glm_4_7_flash/config.py:108-111``).
"""
from __future__ import annotations

import os
from typing import Dict, Optional

import torch
import torch.distributed as dist

from ..ops import reference as R


def padded_tokens(T: int, world: int) -> int:
    """Token count padded so every rank gets an equal, tileable shard."""
    if T <= 256:
        t = 8 * world
        while t < T:
            t *= 2
        if t <= 256:
            return t
    step = 128 * world
    return -(-T // step) * step


def exchange_layout(hidden: int, max_tokens: int, world: int) -> Dict[str, int]:
    """Byte offsets of one rank's exchange buffer, the same for the P2P and NVLS
    flavours: ``ag`` (gathered shards, [N*cap, H] bf16), ``rs`` (P2P: reduce-scatter
    slots [N, cap, H]; NVLS: this rank's full partial output [N*cap, H]), the two
    flag arrays ([N] u32 each), the argmax pairs ([N, am_cap] 8-byte (value, index))
    and their flags.  Every region starts on a 256-byte boundary."""
    al = lambda x: (x + 255) // 256 * 256  # noqa: E731
    N, H = world, hidden
    cap = padded_tokens(max_tokens, world) // world  # rows per rank
    L = {"cap": cap, "ag_off": 0}
    L["rs_off"] = al(N * cap * H * 2)
    L["ag_flag_off"] = al(L["rs_off"] + N * cap * H * 2)
    L["rs_flag_off"] = al(L["ag_flag_off"] + N * 4)
    L["am_cap"] = padded_tokens(max_tokens, world)
    L["am_off"] = al(L["rs_flag_off"] + N * 4)
    L["am_flag_off"] = al(L["am_off"] + N * L["am_cap"] * 8)
    L["total"] = al(L["am_flag_off"] + N * 4)
    return L


class FusedTP:
    """Fused boundaries.  Each rank's exchange buffer holds
    ``gathered [N*cap, H]`` (every rank's normed shard, pushed there by the
    owners' reduce kernels), ``slots [N, cap, H]`` (reduce-scatter partials from
    each source) and the two flag arrays."""

    def __init__(self, hidden: int, max_tokens: int, group=None):
        from ..ops import load_extension
        from .ep import ExchangeBuffer

        self.C = load_extension()
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.H = hidden
        self._set_layout(exchange_layout(hidden, max_tokens, self.world))
        self.buf = ExchangeBuffer(self.total, group)
        self.peers = self.buf.peers
        self.own = self.peers.tolist()[self.rank]
        self.ag_flags_addr = self.own + self.ag_flag_off
        dev = torch.device("cuda", torch.cuda.current_device())
        self.state = torch.zeros(8, dtype=torch.int32, device=dev)
        self.am_state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.gathered = self.C.wrap_bf16(self.own + self.ag_off, self.world * self.cap, hidden)

    def _set_layout(self, L: Dict[str, int]) -> None:
        for k, v in L.items():
            setattr(self, k, v)

    # -------------------------------------------------------------- boundaries
    def publish(self, residual: torch.Tensor, norm_w: torch.Tensor, eps: float, partials: bool,
                x_add: Optional[torch.Tensor] = None, local_out: Optional[torch.Tensor] = None) -> None:
        """residual [pr, H] += x_add (+ sum of partials); rmsnorm(residual) is pushed to every rank."""
        self.C.tp_reduce(self.peers, self.rank, partials, residual.shape[0], self.H, self.ag_off, self.rs_off,
                         self.ag_flag_off, self.rs_flag_off, self.state, x_add, residual, norm_w, eps, local_out)

    def ag_gemm(self, w: torch.Tensor, T: int, swiglu: bool = False) -> torch.Tensor:
        """[T, N_out] = gathered activations @ w^T (w: [N_out, H] or [2*N_out, H] for SwiGLU)."""
        n_out = w.shape[0] // 2 if swiglu else w.shape[0]
        if (swiglu and os.environ.get("MB_SWIGLU_CLUSTER", "0") == "1" and 1 <= T <= 128 and n_out % 64 == 0
                and w.shape[1] % 64 == 0 and w.is_contiguous() and w.dtype == torch.bfloat16):
            from ..ops import native

            return native.swiglu_cluster(self.gathered[:T], w, wait=(self.ag_flags_addr, self.state, self.world))
        fused_swiglu = swiglu and T <= 256 and n_out % 128 == 0
        cols = n_out if fused_swiglu else w.shape[0]
        out = torch.empty(T, cols, dtype=torch.bfloat16, device=w.device)
        x = self.gathered[:T]
        if not swiglu and self._cluster_ok(T, w):
            from ..ops import native

            return native.linear_cluster(x, w, out=out, wait=(self.ag_flags_addr, self.state, self.world))
        ws = torch.empty(16 * T * w.shape[0], dtype=torch.float32, device=w.device) if T <= 256 else None
        if fused_swiglu:  # split-K dual GEMM, SwiGLU after the reduction; waits on the shards' flags
            self.C.swiglu_linear(x, w, out, ws, self.ag_flags_addr, self.state, self.world)
            return out
        self.C.tp_gemm(x, w, out, True, False, False, self.ag_flags_addr, self.state, self.rank, self.world,
                       T // self.world, self.peers, self.rs_off, self.rs_flag_off, ws)
        if swiglu and not fused_swiglu:
            from ..ops import native

            out = native.swiglu(out)
        return out

    def _cluster_ok(self, T: int, w: torch.Tensor) -> bool:
        """Decode-sized gathered GEMMs run as one cluster split-K launch that waits on the shard
        flags itself (no fp32 workspace, no reduction kernel); ``MB_TP_CLUSTER=0`` turns it off."""
        return (os.environ.get("MB_TP_CLUSTER", "1") != "0" and 1 <= T <= 128 and w.dtype == torch.bfloat16
                and w.shape[0] % 128 == 0 and w.shape[1] % 64 == 0 and w.is_contiguous())

    def ag_qkv_rope(self, w, T, q_w, k_w, positions, inv_freq, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot,
                    eps) -> bool:
        """QKV projection of the first T gathered rows with QK-RMSNorm, RoPE and the paged KV write
        in the cluster GEMM's epilogue.  Returns False where the shape is not covered."""
        if D != 128 or w.shape[0] != (Hq + 2 * Hkv) * D or not self._cluster_ok(T, w):
            return False
        from ..ops import native

        native.qkv_rope_cluster(self.gathered[:T], w, q_w, k_w, positions, inv_freq, slots, q_out, k_cache, v_cache,
                                Hq, Hkv, rot, eps, wait=(self.ag_flags_addr, self.state, self.world))
        return True

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor) -> None:
        """Partial [T, H] = x @ w^T, each row stored once into its owner's slot."""
        T = x.shape[0]
        ws = torch.empty(16 * T * w.shape[0], dtype=torch.float32, device=w.device) if T <= 256 else None
        self.C.tp_gemm(x, w, x, False, True, False, 0, self.state, self.rank, self.world, T // self.world,
                       self.peers, self.rs_off, self.rs_flag_off, ws)

    def argmax_exchange(self, vals: torch.Tensor, idxs: torch.Tensor) -> torch.Tensor:
        """Per token row, the (value, global index) pair of this rank's vocabulary slice ->
        the index of the best logit over every rank's slice (P2P pair exchange, one launch)."""
        out = torch.empty(vals.numel(), dtype=torch.long, device=vals.device)
        self.C.tp_argmax_exchange(self.peers, self.rank, self.am_cap, self.am_off, self.am_flag_off, self.am_state,
                                  vals, idxs, out)
        return out

    def gather_rows(self, idx: torch.Tensor, T: int) -> torch.Tensor:
        out = torch.empty(idx.numel(), self.H, dtype=torch.bfloat16, device=idx.device)
        self.C.tp_gather_rows(self.peers, self.rank, T // self.world, self.ag_off, self.ag_flag_off, self.state,
                              idx, out)
        return out


class NvlsTP(FusedTP):
    """NVLS flavour of the fused boundaries (``csrc/cuda/tp_nvls.cu``).

    The exchange buffer is symmetric memory bound to an NVLink multicast object
    (:class:`mod_b200.parallel.symm.SymmetricBuffer`).  The row-parallel GEMM
    writes its whole partial output into this rank's own ``part`` region (a
    plain local GEMM); the boundary kernel then reads each owned row with one
    ``multimem.ld_reduce`` (the NVSwitch sums the ranks' rows), adds the
    residual, applies the next RMSNorm and writes the normed row into every
    rank's ``gathered`` buffer with one ``multimem.st``.  The column-parallel
    GEMMs, the vocabulary-parallel argmax and the row gather are the P2P
    flavour's, run on the same symmetric buffer's unicast peer addresses.

    Cost per boundary and rank: partial rows leave the GPU once (read by the
    switch) and normed rows leave once (replicated by the switch), against N-1
    peer stores of each in the P2P flavour."""

    def __init__(self, hidden: int, max_tokens: int, group=None):
        from ..ops import load_extension
        from .symm import SymmetricBuffer

        self.C = load_extension()
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.H = hidden
        self._set_layout(exchange_layout(hidden, max_tokens, self.world))  # rs region: this rank's partial
        self.buf = SymmetricBuffer(self.total, group)
        self.peers = self.buf.peers
        self.own = self.buf.own
        self.mc = self.buf.mc
        self.ag_flags_addr = self.own + self.ag_flag_off
        dev = torch.device("cuda", torch.cuda.current_device())
        self.state = torch.zeros(8, dtype=torch.int32, device=dev)
        self.am_state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.gathered = self.C.wrap_bf16(self.own + self.ag_off, self.world * self.cap, hidden)

    def publish(self, residual, norm_w, eps, partials, x_add=None, local_out=None) -> None:
        self.C.tp_nvls_reduce(self.own, self.mc, self.rank, self.world, partials, residual.shape[0], 0, True, self.H,
                              self.ag_off, self.rs_off, self.ag_flag_off, self.rs_flag_off, self.state, x_add,
                              residual, norm_w, eps, local_out)

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor) -> None:
        """This rank's partial [T, H] = x @ w^T into its own ``part`` region (local stores only)."""
        from ..ops import native

        T = x.shape[0]
        part = self.C.wrap_bf16(self.own + self.rs_off, T, self.H)
        if T <= 128 and w.shape[0] % 128 == 0 and x.shape[1] % 64 == 0 and x.stride(1) == 1:
            native.linear_cluster(x, w, out=part)
            return
        ws = None
        if T <= 256 and w.shape[0] % 128 == 0:
            splits = 16 if w.shape[0] <= 1024 else 8
            ws = torch.empty(splits * T * w.shape[0], dtype=torch.float32, device=x.device)
        native.linear(x, w, out=part, workspace=ws)

    def close(self) -> None:
        self.buf.close()


def make_tp_comm(kind: str, hidden: int, max_tokens: int, group=None):
    """Boundary implementation by name: ``"p2p"`` (:class:`FusedTP`), ``"nvls"``
    (:class:`NvlsTP`), ``"nccl"`` (:class:`NcclTP`, the library baseline), or
    ``"auto"``: NVLS where every rank's device supports multicast, else P2P."""
    if kind == "auto":
        from .symm import nvls_supported

        kind = "nvls" if nvls_supported(group) else "p2p"
    if kind == "nvls":
        return NvlsTP(hidden, max_tokens, group)
    if kind == "p2p":
        return FusedTP(hidden, max_tokens, group)
    if kind == "nccl":
        return NcclTP(hidden, max_tokens, group)
    raise ValueError(f"unknown tensor-parallel boundary flavour {kind!r} (p2p, nvls, nccl, auto)")


class NcclTP:
    """Baseline: NCCL all-gather / reduce-scatter + cuBLAS, same interface."""

    def __init__(self, hidden: int, max_tokens: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.H = hidden
        self.shard: Optional[torch.Tensor] = None
        self.partial: Optional[torch.Tensor] = None

    def publish(self, residual, norm_w, eps, partials, x_add=None, local_out=None):
        if partials:
            if dist.get_backend(self.group) == "nccl":
                red = torch.empty_like(residual)
                dist.reduce_scatter_tensor(red, self.partial.contiguous(), group=self.group)
            else:  # gloo has no reduce-scatter: all-reduce and keep this rank's rows
                full = self.partial.clone()
                dist.all_reduce(full, group=self.group)
                pr = residual.shape[0]
                red = full[self.rank * pr:(self.rank + 1) * pr]
            residual.add_(red.to(residual.dtype))
        if x_add is not None:
            residual.add_(x_add)
        self.shard = R.rmsnorm(residual, norm_w, eps)
        if local_out is not None:
            local_out.copy_(self.shard)

    def _gather(self, T):
        parts = [torch.empty_like(self.shard) for _ in range(self.world)]
        dist.all_gather(parts, self.shard.contiguous(), group=self.group)
        return torch.cat(parts, 0)

    def ag_gemm(self, w, T, swiglu=False):
        y = torch.matmul(self._gather(T), w.t())
        return R.swiglu(y) if swiglu else y

    def gemm_rs(self, x, w):
        self.partial = torch.matmul(x, w.t())

    def gather_rows(self, idx, T):
        return self._gather(T).index_select(0, idx)


class FusedVisionExchange:
    """Vision -> LLM rows over NVLink: the merger's last linear runs as a GEMM
    whose epilogue adds the bias and stores each visual row into its owner's
    buffer (P2P), the last CTA releasing a flag at every rank; the owner waits
    for every rank's flag and copies the rows of its shard that hold image
    tokens into its embeddings.  A rank with no visual rows only releases."""

    def __init__(self, hidden: int, max_tokens: int, group=None):
        from ..ops import load_extension
        from .ep import ExchangeBuffer

        self.C = load_extension()
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.H = hidden
        self.cap = padded_tokens(max_tokens, self.world) // self.world
        al = lambda x: (x + 255) // 256 * 256  # noqa: E731
        self.off = 0
        self.flag_off = al(self.cap * hidden * 2)
        self.buf = ExchangeBuffer(al(self.flag_off + self.world * 4), group)
        self.peers = self.buf.peers
        self.state = torch.zeros(8, dtype=torch.int32, device=torch.device("cuda", torch.cuda.current_device()))

    def exchange(self, x, w, bias, row_map, h_shard, my_rows, pr: int) -> None:
        assert pr <= self.cap, "step larger than the exchange capacity"
        if x.shape[0] > 0:
            self.C.vis_scatter_gemm(x, w, bias, row_map, self.peers, self.rank, pr, self.off, self.flag_off,
                                    self.state)
        else:
            self.C.vis_release(self.peers, self.rank, self.flag_off, self.state)
        self.C.vis_wait_merge(self.peers, self.rank, self.off, self.flag_off, self.state, my_rows, h_shard)


class NcclVisionExchange:
    """Baseline: every rank computes its rows' merger output, the (row, value)
    lists are all-gathered with the process group, each rank keeps its shard's."""

    def __init__(self, backend, group=None):
        self.be, self.group = backend, group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def exchange(self, x, w, bias, row_map, h_shard, my_rows, pr: int) -> None:
        H = w.shape[0]
        y = self.be.linear(x, w, bias=bias) if x.shape[0] else torch.empty(0, H, dtype=h_shard.dtype, device=x.device)
        n = torch.tensor([y.shape[0]], device=x.device)
        ns = [torch.zeros_like(n) for _ in range(self.world)]
        dist.all_gather(ns, n, group=self.group)
        m = max(int(v.item()) for v in ns)
        if m == 0:
            return
        yp = torch.zeros(m, H, dtype=h_shard.dtype, device=x.device)
        rp = torch.full((m,), -1, dtype=torch.int32, device=x.device)
        yp[:y.shape[0]] = y.to(h_shard.dtype)
        rp[:y.shape[0]] = row_map
        ys = [torch.empty_like(yp) for _ in range(self.world)]
        rs = [torch.empty_like(rp) for _ in range(self.world)]
        dist.all_gather(ys, yp, group=self.group)
        dist.all_gather(rs, rp, group=self.group)
        ya, ra = torch.cat(ys), torch.cat(rs).long()
        keep = (ra >= self.rank * pr) & (ra < (self.rank + 1) * pr)
        h_shard[ra[keep] - self.rank * pr] = ya[keep]
