"""Gated DeltaNet linear attention (Qwen3-Next), engine path.

Math (per value head, state S in R^{dk x dv}):
    S_t = exp(g_t) * S_{t-1}
    S_t = S_t + k_t (beta_t * (v_t - S_t^T k_t))^T
    o_t = S_t^T q_t
with q, k L2-normalised (q also scaled by dk^-1/2), beta = sigmoid(b),
g = -exp(A_log) * softplus(a + dt_bias).  Inputs pass through a causal
depthwise conv (kernel 4) + SiLU; the output goes through a gated RMSNorm
(norm(o) * w * silu(z)) and the out projection.

Prefill uses the chunked form of the delta rule (Yang, Kautz, Hatamizadeh,
"Gated Delta Networks", 2024): within a chunk of C tokens the sequential
updates collapse to a unit-lower-triangular solve (the WY/UT representation),
so the work becomes C x C and C x d matrix products; a state recurrence links
the chunks.  Decode applies one recurrent step per sequence.

The reference implements a decayed linear attention instead
(``pio/plugins/cpu/c_src/tensor_ops.c:780-811``,
``pio/models/qwen3_coder_next/model.py:231-277``).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _l2n(x):
    return x * torch.rsqrt(x.pow(2).sum(-1, keepdim=True) + 1e-6)


def chunk_gated_delta_rule(q, k, v, g, beta, state, chunk: int = 64):
    """q, k: [H, L, dk]; v: [H, L, dv]; g, beta: [H, L]; state: [H, dk, dv] (fp32).
    Returns (o [H, L, dv], new state)."""
    H, L, dk = q.shape
    dv = v.shape[-1]
    pad = (-L) % chunk
    if pad:
        q = F.pad(q, (0, 0, 0, pad))
        k = F.pad(k, (0, 0, 0, pad))
        v = F.pad(v, (0, 0, 0, pad))
        g = F.pad(g, (0, pad))
        beta = F.pad(beta, (0, pad))
    n = q.shape[1] // chunk
    q, k, v = (t.reshape(H, n, chunk, -1) for t in (q, k, v))
    g = g.reshape(H, n, chunk).cumsum(-1)                       # cumulative log-decay inside a chunk
    beta = beta.reshape(H, n, chunk)
    kb = k * beta[..., None]
    vb = v * beta[..., None]
    tri = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device)
    lower_strict = tri.tril(-1)
    lower = tri.tril()
    decay = torch.exp((g[..., :, None] - g[..., None, :]).masked_fill(~lower, -float("inf")))
    # A = (I + strict_lower(diag(beta) K K^T * decay))^{-1}, by forward substitution
    M = (kb @ k.transpose(-1, -2)) * decay
    M = M.masked_fill(~lower_strict, 0.0)
    eye = torch.eye(chunk, device=q.device, dtype=q.dtype)
    A = torch.linalg.solve_triangular(eye + M, eye.expand_as(M), upper=False, unitriangular=True)
    u = A @ vb                                                   # pseudo-values
    w = A @ (kb * torch.exp(g)[..., None])                       # decayed keys
    o = torch.empty_like(v)
    S = state
    causal = (q @ k.transpose(-1, -2)) * decay                   # [H, n, C, C], lower incl. diagonal
    for c in range(n):
        v_new = u[:, c] - w[:, c] @ S
        o[:, c] = (q[:, c] * torch.exp(g[:, c])[..., None]) @ S + causal[:, c] @ v_new
        gl = g[:, c, -1]
        S = S * torch.exp(gl)[:, None, None] + (k[:, c] * torch.exp(gl[:, None] - g[:, c])[..., None]).transpose(
            -1, -2) @ v_new
    o = o.reshape(H, n * chunk, dv)[:, :L]
    return o, S


def recurrent_step(q, k, v, g, beta, state):
    """One token per sequence.  q,k: [B, H, dk], v: [B, H, dv], g, beta: [B, H], state [B, H, dk, dv]."""
    state = state * torch.exp(g)[..., None, None]
    kv = torch.einsum("bhkv,bhk->bhv", state, k)
    delta = (v - kv) * beta[..., None]
    state = state + torch.einsum("bhk,bhv->bhkv", k, delta)
    o = torch.einsum("bhkv,bhk->bhv", state, q)
    return o, state


def _gates(ba, A_log, dt_bias, Hv):
    ba = ba.float()
    beta = torch.sigmoid(ba[:, :Hv])
    g = -torch.exp(A_log.float()) * F.softplus(ba[:, Hv:] + dt_bias.float())
    return beta, g


def _split_qkv(mixed, Hk, Hv, dk, dv):
    kd = Hk * dk
    T = mixed.shape[0]
    q = mixed[:, :kd].reshape(T, Hk, dk)
    k = mixed[:, kd:2 * kd].reshape(T, Hk, dk)
    v = mixed[:, 2 * kd:].reshape(T, Hv, dv)
    rep = Hv // Hk
    q = _l2n(q).repeat_interleave(rep, dim=1) / math.sqrt(dk)
    k = _l2n(k).repeat_interleave(rep, dim=1)
    return q, k, v


def _gated_norm(o, z, norm_w, eps, Hv, dv):
    T = o.shape[0]
    zf = z.float().reshape(T, Hv, dv)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()
    return (o * F.silu(zf)).reshape(T, Hv * dv)


def ref_prefill(mix, z, ba, conv_w, A_log, dt_bias, norm_w, conv_state, ssm_state, slot: int, Hk, Hv, dk, dv, eps):
    """fp32 oracle of one sequence's prefill after the projections (mix = raw q|k|v channels).
    Updates ``conv_state[slot]`` / ``ssm_state[slot]``; returns the gated-normed output [L, Hv*dv] fp32."""
    beta, g = _gates(ba, A_log, dt_bias, Hv)
    Kc = conv_w.shape[1]
    xin = torch.cat([conv_state[slot].t(), mix.float()], dim=0)        # [K-1+L, C]
    conv_state[slot] = xin[-(Kc - 1):].t()
    xc = F.conv1d(xin.t()[None], conv_w.float()[:, None, :], groups=xin.shape[1])[0].t()
    q, k, v = _split_qkv(F.silu(xc), Hk, Hv, dk, dv)
    o, S = chunk_gated_delta_rule(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1).float(),
                                  g.t(), beta.t(), ssm_state[slot])
    ssm_state[slot] = S
    return _gated_norm(o.transpose(0, 1), z, norm_w, eps, Hv, dv)


def ref_decode(mix, z, ba, conv_w, A_log, dt_bias, norm_w, conv_state, ssm_state, slots, Hk, Hv, dk, dv, eps):
    """fp32 oracle of one decode step (one token per sequence in ``slots``)."""
    beta, g = _gates(ba, A_log, dt_bias, Hv)
    cs = conv_state[slots]                                           # [B, C, K-1]
    xin = torch.cat([cs, mix.float()[:, :, None]], dim=2)            # [B, C, K]
    conv_state[slots] = xin[:, :, 1:]
    q, k, v = _split_qkv(F.silu((xin * conv_w.float()[None]).sum(-1)), Hk, Hv, dk, dv)
    o, S = recurrent_step(q, k, v.float(), g, beta, ssm_state[slots])
    ssm_state[slots] = S
    return _gated_norm(o, z, norm_w, eps, Hv, dv)


class DeltaNetLayer:
    """Engine-side gated DeltaNet block.  ``be`` supplies the GEMMs."""

    def __init__(self, cfg, dw, num_k_heads=None, num_v_heads=None):
        self.cfg, self.w = cfg, dw
        self.Hk = num_k_heads or cfg.linear_num_key_heads
        self.Hv = num_v_heads or cfg.linear_num_value_heads
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self._f32 = None

    def _native(self, be, x) -> bool:
        return (getattr(be, "name", "") == "native" and x.dtype == torch.bfloat16 and self.dk == self.dv
                and self.dk in (64, 128) and self.w.conv.shape[1] == 4 and self.Hv % self.Hk == 0)

    def _gates_f32(self):
        if self._f32 is None:
            self._f32 = (self.w.A_log.float().contiguous(), self.w.dt_bias.float().contiguous(),
                         self.w.conv.to(torch.bfloat16).contiguous(), self.w.norm.to(torch.bfloat16).contiguous())
        return self._f32

    def _native_split(self, be, x):
        kd, vd = self.Hk * self.dk, self.Hv * self.dv
        p = be.linear(x, self.w.in_qkvz)
        ba = be.linear(x, self.w.in_ba)
        return p[:, :2 * kd + vd].contiguous(), p[:, 2 * kd + vd:].contiguous(), ba.contiguous()

    def decode_native(self, be, x, conv_state, ssm_state, slots):
        """Fused decode kernel (conv, norms, gates, delta rule, gated RMSNorm), then out projection."""
        mixed, z, ba = self._native_split(be, x)
        A, dtb, cw, nw = self._gates_f32()
        o = be.N.deltanet_decode(mixed, z, ba, cw, conv_state, ssm_state, slots, A, dtb, nw, self.Hk, self.Hv,
                                 self.dk, self.dv, self.cfg.rms_norm_eps)
        return be.linear(o, self.w.out)

    def prefill_native(self, be, x, conv_state, ssm_state, slots, query_lens):
        """All prefill sequences of a step in one conv kernel + one scan kernel."""
        mixed, z, ba = self._native_split(be, x)
        A, dtb, cw, nw = self._gates_f32()
        ql = torch.tensor(query_lens, dtype=torch.int32)
        cu = torch.zeros(len(query_lens) + 1, dtype=torch.int32)
        cu[1:] = ql.cumsum(0)
        seq_of = torch.repeat_interleave(torch.arange(len(query_lens), dtype=torch.int32), ql)
        dev = x.device
        o = be.N.deltanet_prefill(mixed, z, ba, cw, conv_state, ssm_state, slots, cu.to(dev), seq_of.to(dev), A,
                                  dtb, nw, self.Hk, self.Hv, self.dk, self.dv, self.cfg.rms_norm_eps)
        return be.linear(o, self.w.out)

    def core(self, be, mixed, z, ba, conv_state, ssm_state, fb):
        """Conv, gates, delta rule and gated RMSNorm from already projected inputs (mixed q|k|v
        channels, z, beta/decay logits) for every sequence of the step; returns the rows that
        go into the output projection.  Tensor parallelism calls it with this rank's heads."""
        if self._native(be, mixed):
            A, dtb, cw, nw = self._gates_f32()
            mixed, z, ba = mixed.contiguous(), z.contiguous(), ba.contiguous()
            if fb.is_decode:
                return be.N.deltanet_decode(mixed, z, ba, cw, conv_state, ssm_state, fb.state_slots, A, dtb, nw,
                                            self.Hk, self.Hv, self.dk, self.dv, self.cfg.rms_norm_eps)
            ql = torch.tensor(fb.query_lens, dtype=torch.int32)
            cu = torch.zeros(len(fb.query_lens) + 1, dtype=torch.int32)
            cu[1:] = ql.cumsum(0)
            seq_of = torch.repeat_interleave(torch.arange(len(fb.query_lens), dtype=torch.int32), ql)
            dev = mixed.device
            return be.N.deltanet_prefill(mixed, z, ba, cw, conv_state, ssm_state, fb.state_slots, cu.to(dev),
                                         seq_of.to(dev), A, dtb, nw, self.Hk, self.Hv, self.dk, self.dv,
                                         self.cfg.rms_norm_eps)
        w = self.w
        if fb.is_decode:
            o = ref_decode(mixed, z, ba, w.conv, w.A_log, w.dt_bias, w.norm, conv_state, ssm_state, fb.state_slots,
                           *self._dims())
            return o.to(mixed.dtype)
        outs, start = [], 0
        for b, ql in enumerate(fb.query_lens):
            sl = slice(start, start + ql)
            outs.append(ref_prefill(mixed[sl], z[sl], ba[sl], w.conv, w.A_log, w.dt_bias, w.norm, conv_state,
                                    ssm_state, int(fb.state_slots[b]), *self._dims()))
            start += ql
        return torch.cat(outs, 0).to(mixed.dtype)

    def _dims(self):
        return self.Hk, self.Hv, self.dk, self.dv, self.cfg.rms_norm_eps

    def prefill(self, be, x, conv_state, ssm_state, slot: int):
        """x: [L, H] tokens of one sequence; updates the slot's states in place."""
        mix, z, ba = self._native_split(be, x)
        w = self.w
        o = ref_prefill(mix, z, ba, w.conv, w.A_log, w.dt_bias, w.norm, conv_state, ssm_state, slot, *self._dims())
        return be.linear(o.to(x.dtype), w.out)

    def decode(self, be, x, conv_state, ssm_state, slots):
        """x: [B, H], one token per sequence in ``slots``."""
        mix, z, ba = self._native_split(be, x)
        w = self.w
        o = ref_decode(mix, z, ba, w.conv, w.A_log, w.dt_bias, w.norm, conv_state, ssm_state, slots, *self._dims())
        return be.linear(o.to(x.dtype), w.out)
