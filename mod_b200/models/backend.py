"""Op backends the model layers call.

* :class:`NativeBackend`  - the product path: sm_100a kernels from ``mod_b200._C``.
* :class:`TorchBackend`   - the baseline: PyTorch ops, cuBLAS GEMMs (``torch.matmul``),
  SDPA attention.  Also runs on CPU, where it backs the CPU tests.

Both take and return bf16 tensors and the same buffer conventions, so a model
switches paths with one constructor argument.  The reference's equivalent is
the ctypes ``Tensor`` method table (``pio/core/engine/backend.py:332-654``).
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

from ..ops import reference as R
from ..ops.quant import Int8Weight, dense


class TorchBackend:
    name = "torch"

    def linear(self, x, w, bias=None, residual=None, out=None):
        y = R.linear(x, dense(w, x.dtype), residual=residual)
        if bias is not None:
            y = y + bias
        if out is not None:
            out.copy_(y)
            return out
        return y

    def rmsnorm(self, x, w, eps, residual=None):
        return R.rmsnorm(x, w, eps, residual=residual)

    def linear_gelu(self, x, w, bias=None):
        y = R.linear(x, dense(w, x.dtype)).float()
        if bias is not None:
            y = y + bias.float()
        return F.gelu(y, approximate="tanh").to(x.dtype)

    def swiglu_mlp(self, x, gate_up, down, residual=None):
        h = R.swiglu(R.linear(x, dense(gate_up, x.dtype)))
        return R.linear(h, dense(down, x.dtype), residual=residual)

    def rope_qknorm(self, qkv, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot, eps):
        return R.rope_qknorm(qkv, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot, eps)

    def attn_decode(self, q, k_cache, v_cache, block_tables, ctx_lens, splits=1):
        return R.attn_decode_batched(q, k_cache, v_cache, block_tables, ctx_lens)

    def attn_prefill(self, q, k, v):
        return R.attn_prefill(q, k, v)

    def moe(self, x, mo, top_k, renorm, inter, residual=None):
        """Full routed-expert block on all experts held by this process."""
        logits = R.linear(x, mo.router)
        ids, wts = R.moe_route(logits, top_k, renorm)
        E = mo.e_hi - mo.e_lo
        out = R.moe_experts(x, ids - mo.e_lo, wts, dense(mo.w13, x.dtype), dense(mo.w2, x.dtype), E, inter)
        if mo.shared is not None:
            sh = self.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down).float()
            out = out + torch.sigmoid(R.linear(x, mo.shared_gate).float()) * sh
        if residual is not None:
            out = out + residual.float()
        return out.to(x.dtype)

    def embed(self, ids, table):
        return R.embed(ids, table)

    def argmax(self, logits):
        return R.argmax(logits)


class NativeBackend:
    """sm_100a kernels.  Scratch tensors come from the caching allocator, so a
    captured CUDA graph owns them through its private memory pool."""

    name = "native"

    def __init__(self):
        from ..ops import native as N
        from ..ops import load_extension

        load_extension()
        self.N = N
        self._one_group = {}
        # MB_CLUSTER_GEMM=0 keeps decode GEMMs on the split-K + reduction kernels (A/B timing)
        self.cluster_gemm = os.environ.get("MB_CLUSTER_GEMM", "1") != "0"
        # int8 weights on the cluster kernel are opt-in (MB_CLUSTER_W8=1): its in-loop expansion measured
        # slower than the int8 split-K kernel at T = 128 (33.3 vs 30.4 us, Qwen3-30B-A3B qkv)
        self.cluster_w8 = os.environ.get("MB_CLUSTER_W8", "0") == "1"

    def _sms(self, device) -> int:
        if not hasattr(self, "_nsm"):
            self._nsm = torch.cuda.get_device_properties(device).multi_processor_count
        return self._nsm

    def _offs1(self, T, device):
        # built by a kernel (no host copy), so it is legal inside graph capture
        return torch.arange(2, dtype=torch.int32, device=device) * T

    def _cluster_ok(self, x2, w) -> bool:
        """Decode-sized GEMMs (bf16 or int8 weights) run on the cluster split-K kernel (DSMEM
        reduction, one launch)."""
        if not self.cluster_gemm or x2.dtype != torch.bfloat16:
            return False
        if isinstance(w, Int8Weight) and not self.cluster_w8:
            return False
        wt = w.q if isinstance(w, Int8Weight) else w
        if wt.dtype not in (torch.bfloat16, torch.int8):
            return False
        T, K = x2.shape
        return (1 <= T <= 128 and wt.shape[0] % 128 == 0 and wt.shape[0] <= 16384 and K % 64 == 0
                and x2.stride(1) == 1 and wt.is_contiguous())

    def linear(self, x, w, bias=None, residual=None, out=None):
        x2 = x.reshape(-1, x.shape[-1])
        if bias is None and self._cluster_ok(x2, w) and (out is None or out.is_contiguous()):
            o = None if out is None else out.view(x2.shape[0], w.shape[0])
            r = None if residual is None else residual.reshape(x2.shape[0], -1)
            if isinstance(w, Int8Weight):
                y = self.N.linear_cluster_w8(x2, w.q, w.scale, out=o, residual=r)
            else:
                y = self.N.linear_cluster(x2, w, out=o, residual=r)
            return y if out is None else out
        T = x2.shape[0]
        ws = None
        n_out = w.shape[0]
        max_splits = 16 if n_out <= 1024 else (8 if n_out <= 128 * self._sms(x.device) else 0)
        if T <= 256 and n_out % 128 == 0 and max_splits:
            # split-K workspace for skinny (decode) shapes that can split (not the LM head)
            ws = torch.empty(max_splits * T * n_out, dtype=torch.float32, device=x.device)
        if isinstance(w, Int8Weight):
            if w.shape[0] % 128 == 0 and w.shape[1] % 64 == 0:
                y = self.N.linear_w8(x, w.q, w.scale, out=out, residual=residual, workspace=ws)
            else:  # shapes outside the kernel's tiling
                y = self.N.linear(x, w.dequant(x.dtype), out=out, residual=residual)
        else:
            y = self.N.linear(x, w, out=out, residual=residual, workspace=ws)
        if bias is not None:
            if y.dim() == 2 and y.shape[1] % 8 == 0 and y.is_contiguous():
                self.N.bias_act(y, bias, False)
            else:
                y += bias
        return y

    def linear_gelu(self, x, w, bias=None):
        """tanh-GELU(x @ w^T + bias): GEMM, then one fused bias + activation pass."""
        y = self.N.linear(x, w) if not isinstance(w, Int8Weight) else self.linear(x, w)
        if y.shape[1] % 8 == 0:
            return self.N.bias_act(y, bias, True)
        y = y.float() + (bias.float() if bias is not None else 0)
        return F.gelu(y, approximate="tanh").to(x.dtype)

    def rmsnorm(self, x, w, eps, residual=None):
        return self.N.rmsnorm(x, w, eps, residual=residual)

    def swiglu_mlp(self, x, gate_up, down, residual=None):
        x2 = x.reshape(-1, x.shape[-1])
        T = x2.shape[0]
        I = gate_up.shape[0] // 2
        if isinstance(gate_up, Int8Weight):
            if I % 128 == 0 and gate_up.shape[1] % 64 == 0:
                ws = torch.empty(8 * T * 2 * I, dtype=torch.float32, device=x.device) if T <= 256 else None
                h = self.N.linear_w8(x2, gate_up.q, gate_up.scale, workspace=ws, swiglu=True)
            else:
                h = self.N.swiglu(self.linear(x2, gate_up))
        elif (T <= 128 and I % 64 == 0 and x2.shape[1] % 64 == 0 and gate_up.is_contiguous()
              and os.environ.get("MB_SWIGLU_CLUSTER", "0") == "1"):
            h = self.N.swiglu_cluster(x2, gate_up)   # one cluster launch (opt-in until measured)
        elif I % 128 == 0 and T <= 256:
            h = self.N.swiglu_linear(x2, gate_up)
        elif I % 128 == 0:
            offs = self._offs1(T, x.device)
            h = self.N.grouped_linear(x2, gate_up, offs, 1, True, T)
        else:
            h = self.N.swiglu(self.linear(x2, gate_up))
        return self.linear(h, down, residual=residual)

    def rope_qknorm(self, qkv, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot, eps):
        return self.N.rope_qknorm(qkv, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot,
                                  eps)

    def qkv_rope(self, x, w, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot, eps) -> bool:
        """QKV projection with QK-norm, RoPE and the KV write in one cluster GEMM (decode sizes,
        head_dim 128).  Returns False when the shape is not covered (caller runs the two-step form)."""
        if (D != 128 or isinstance(w, Int8Weight) or w.shape[0] != (Hq + 2 * Hkv) * D
                or not self._cluster_ok(x, w)):
            return False
        self.N.qkv_rope_cluster(x, w, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, rot, eps)
        return True

    def attn_decode(self, q, k_cache, v_cache, block_tables, ctx_lens, splits=1):
        B, Hq, D = q.shape
        tc = self.N.attn_decode_tc_supported(D, Hq // k_cache.shape[1])
        impl = os.environ.get("MB_ATTN_IMPL", "tc")  # A/B timing: "cuda" forces the CUDA-core kernel
        tc = tc and impl != "cuda"
        dynamic = os.environ.get("MB_ATTN_DYNAMIC", "1") != "0"
        chunk_env = os.environ.get("MB_ATTN_CHUNK")
        if tc:
            # persistent tcgen05 kernel (3 CTAs per SM) with a dynamic work queue (longest items first);
            # sequences are cut into chunks of 16 blocks only when (sequence, KV head) items do not
            # fill the resident CTAs.
            # measured (Qwen3-30B-A3B shapes, ctx 600): 128 sequences x 4 KV heads run fastest unsplit
            # (50.7 us vs 68-89 us with any split: the split-KV partials and combine cost more than the
            # imbalance); 16 sequences run fastest in chunks of 16 blocks (17.3 vs 22.4 us unsplit)
            mb = block_tables.shape[1]
            items = B * k_cache.shape[1]
            chunk = mb if items >= 3 * self._sms(q.device) else 16
            if chunk_env is not None:  # blocks per chunk; 0 = whole sequences
                chunk = int(chunk_env) or mb
            splits = max(1, -(-mb // chunk))
        elif chunk_env is not None:
            splits = max(1, -(-block_tables.shape[1] // (int(chunk_env) or block_tables.shape[1])))
        ws = None
        if splits > 1:
            ws = torch.empty(B * Hq * splits * (D + 1), dtype=torch.float32, device=q.device)
        if tc:
            return self.N.attn_decode_tc(q, k_cache, v_cache, block_tables, ctx_lens, splits=splits, workspace=ws,
                                         dynamic=dynamic)
        return self.N.attn_decode(q, k_cache, v_cache, block_tables, ctx_lens, splits=splits, workspace=ws)

    def attn_prefill(self, q, k, v):
        return R.attn_prefill(q, k, v)

    def attn_prefill_paged(self, q, k_cache, v_cache, fb):
        """All sequences of a prefill step in one tcgen05 flash-attention launch
        (head_dim 64, 128 or 256); None when the shape is not covered."""
        if q.shape[-1] not in (64, 128, 256):
            return None
        ql = fb.query_lens
        cu = [0]
        for n in ql:
            cu.append(cu[-1] + n)
        cu_q = torch.tensor(cu, dtype=torch.int32).to(q.device, non_blocking=True)
        return self.N.attn_prefill_tc(q, k_cache, v_cache, fb.block_tables, cu_q, fb.ctx_lens, max(ql))

    def moe(self, x, mo, top_k, renorm, inter, residual=None):
        N = self.N
        T, H = x.shape
        E = mo.router.shape[0]
        dev = x.device
        logits = self.linear(x, mo.router)
        ids = torch.empty(T, top_k, dtype=torch.int32, device=dev)
        wts = torch.empty(T, top_k, dtype=torch.float32, device=dev)
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        offs = torch.empty(E + 1, dtype=torch.int32, device=dev)
        cursor = torch.empty(E, dtype=torch.int32, device=dev)
        N.moe_route(logits, top_k, renorm, ids, wts, counts, offs, cursor)
        pos = torch.empty(T, top_k, dtype=torch.int32, device=dev)
        xs = torch.empty(T * top_k, H, dtype=x.dtype, device=dev)
        N.moe_permute(x, ids, offs, cursor, pos, xs)
        exp_rows = max(1, (T * top_k) // E)
        max_rows = min(T * top_k, 4 * exp_rows)
        if isinstance(mo.w13, Int8Weight):
            h = N.linear_w8(xs, mo.w13.q, mo.w13.scale, offs=offs, groups=E, swiglu=True, max_rows_per_group=max_rows)
        else:
            h = N.grouped_linear(xs, mo.w13, offs, E, True, max_rows)
        if isinstance(mo.w2, Int8Weight):
            y = N.linear_w8(h, mo.w2.q, mo.w2.scale, offs=offs, groups=E, max_rows_per_group=max_rows)
        else:
            y = N.grouped_linear(h, mo.w2, offs, E, False, max_rows)
        out = torch.empty_like(x)
        if mo.shared is not None:
            sh = self.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down)
            # [T, 1] gate: a GEMV too narrow for a tensor-core tile
            g = torch.sigmoid((x.float() @ mo.shared_gate.float().t()))
            res2 = (sh.float() * g + (residual.float() if residual is not None else 0)).to(x.dtype)
            return N.moe_combine(y, pos, wts, res2, out)
        return N.moe_combine(y, pos, wts, residual, out)

    def embed(self, ids, table):
        return self.N.embed(ids, table)

    def argmax(self, logits):
        return self.N.argmax(logits.contiguous())


def _rows_f32(w, lo: int, hi: int) -> torch.Tensor:
    """Rows [lo, hi) of a weight (fp32 / bf16 tensor or Int8Weight) as fp32."""
    if isinstance(w, Int8Weight):
        return w.q[lo:hi].float() * w.scale[lo:hi, None].float()
    return w[lo:hi].float()


class CpuBackend(TorchBackend):
    """C++/OpenMP CPU backend (``mod_b200._cpu``), fp32.  Plumbing and host
    reference path; the reference's equivalent is its C CPU library
    (``pio/plugins/cpu/c_src/tensor_ops.c``)."""

    name = "cpu"

    def linear_gelu(self, x, w, bias=None):
        return F.gelu(self.linear(x, w, bias=bias).float(), approximate="tanh").to(x.dtype)

    def __init__(self, threads: Optional[int] = None):
        import importlib

        self.C = importlib.import_module("mod_b200._cpu")
        if threads:
            self.C.set_num_threads(threads)

    def linear(self, x, w, bias=None, residual=None, out=None):
        x2 = x.reshape(-1, x.shape[-1]).float().contiguous()
        y = torch.empty(x2.shape[0], w.shape[0], dtype=torch.float32)
        if isinstance(w, Int8Weight):   # int8 weight-only: widened in registers, per-channel scale
            self.C.linear_w8(x2, w.q.contiguous(), w.scale.float().contiguous(), y)
        else:
            # bf16 weights stay bf16 (widened in registers: half the weight bytes); others go to fp32
            if not (isinstance(w, torch.Tensor) and w.dtype == torch.bfloat16 and w.is_contiguous()):
                w = dense(w, torch.float32)
            self.C.linear(x2, w, y)
        if bias is not None:
            y += bias
        if residual is not None:
            y += residual.reshape(y.shape)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def rmsnorm(self, x, w, eps, residual=None):
        out = torch.empty_like(x)
        self.C.rmsnorm(x.contiguous(), residual, w.float(), out, eps)
        return out

    def swiglu_mlp(self, x, gate_up, down, residual=None):
        gu = self.linear(x, gate_up)
        h = torch.empty(gu.shape[0], gu.shape[1] // 2)
        self.C.swiglu(gu, h)
        return self.linear(h, down, residual=residual)

    def rope_qknorm(self, qkv, q_w, k_w, positions, invf, slots, q_out, k_cache, v_cache, Hq, Hkv, D, rot, eps):
        self.C.rope_qknorm(qkv.contiguous(), None if q_w is None else q_w.float(),
                           None if k_w is None else k_w.float(), positions, invf, slots, q_out, k_cache, v_cache, Hq,
                           Hkv, D, rot, eps)
        return q_out

    def attn_paged(self, q, k_cache, v_cache, fb):
        out = torch.empty_like(q)
        if fb.is_decode:
            qlens = torch.ones(q.shape[0], dtype=torch.int32)
        else:
            qlens = torch.tensor(fb.query_lens, dtype=torch.int32)
        self.C.attn_paged(q, k_cache, v_cache, fb.block_tables, fb.ctx_lens, qlens, out, 1.0 / math.sqrt(q.shape[-1]))
        return out

    def moe(self, x, mo, top_k, renorm, inter, residual=None):
        logits = self.linear(x, mo.router)
        T = x.shape[0]
        ids = torch.empty(T, top_k, dtype=torch.int32)
        wts = torch.empty(T, top_k)
        self.C.moe_route(logits, top_k, renorm, ids, wts)
        out = torch.zeros_like(x) if residual is None else residual.clone()
        E_l = mo.e_hi - mo.e_lo
        if isinstance(mo.w13, torch.Tensor) and mo.w13.dtype == torch.float32:
            self.C.moe_experts(x.contiguous(), ids, wts, mo.w13, mo.w2, mo.e_lo, E_l, out)
        else:
            # narrow (bf16 / int8) experts: widen only the experts this call routes to, then run the
            # same fp32 expert kernel on the compacted set (ids remapped; others skipped as -1)
            local = ids.long() - mo.e_lo
            active = torch.unique(local[(local >= 0) & (local < E_l)])
            if active.numel():
                remap = torch.full((E_l,), -1, dtype=torch.long)
                remap[active] = torch.arange(active.numel())
                cids = torch.where((local >= 0) & (local < E_l), remap[local.clamp(0, E_l - 1)],
                                   torch.full_like(local, -1)).to(torch.int32)
                r13, r2 = mo.w13.shape[0] // E_l, mo.w2.shape[0] // E_l
                w13c = torch.cat([_rows_f32(mo.w13, int(e) * r13, (int(e) + 1) * r13) for e in active])
                w2c = torch.cat([_rows_f32(mo.w2, int(e) * r2, (int(e) + 1) * r2) for e in active])
                self.C.moe_experts(x.contiguous(), cids, wts, w13c.contiguous(), w2c.contiguous(), 0,
                                   int(active.numel()), out)
        if mo.shared is not None:
            sh = self.swiglu_mlp(x, mo.shared.gate_up, mo.shared.down)
            out += torch.sigmoid(x.float() @ mo.shared_gate.float().t()) * sh
        return out

    def embed(self, ids, table):
        if table.dtype != torch.float32:  # bf16 table: gather the rows, widen only those
            return table[ids.reshape(-1).long()].float()
        out = torch.empty(ids.numel(), table.shape[1])
        self.C.embed(ids.contiguous(), table, out)
        return out

    def argmax(self, logits):
        return self.C.argmax(logits.float().contiguous())


def make_backend(name: str):
    if name == "native":
        return NativeBackend()
    if name == "cpu":
        return CpuBackend()
    if name in ("torch", "baseline", "reference"):
        return TorchBackend()
    raise ValueError(f"unknown backend {name!r}")
