"""fp32 numerical oracle: a direct PyTorch statement of the correct architectures.

It recomputes the whole sequence with no cache (causal attention, GQA,
per-head QK-RMSNorm, RoPE, SwiGLU/GELU MLP, softmax top-k MoE with
renormalisation and optional shared expert, gated DeltaNet as a sequential
recurrence).  The reference cannot serve as oracle: its attention is not
causal, its Qwen3 attention has the wrong head_dim and no QK-norm, and its
DeltaNet is a decayed linear attention (``pio/plugins/cpu/c_src/tensor_ops.c:536-578``,
``pio/models/qwen3_0_6b/architecture.py:39-47``, ``pio/models/qwen3_coder_next/model.py:261-271``).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..config.models import ModelConfig
from ..ops import reference as R
from .weights import ModelWeights


def _f(t):
    return None if t is None else t.float()


def rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def attention_block(cfg: ModelConfig, aw, x, pos):
    B, S, H = x.shape
    Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    qkv = x @ _f(aw.qkv).t()
    if aw.qkv_bias is not None:
        qkv = qkv + _f(aw.qkv_bias)
    q = qkv[..., : Hq * D].reshape(B, S, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hkv) * D].reshape(B, S, Hkv, D)
    v = qkv[..., (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].reshape(B, S, Hkv, D)
    if aw.q_norm is not None:
        q = rms(q, _f(aw.q_norm), cfg.rms_norm_eps)
        k = rms(k, _f(aw.k_norm), cfg.rms_norm_eps)
    invf = R.inv_freq(cfg.rotary_dim, cfg.rope_theta, device=x.device)
    q = torch.stack([R.apply_rope(q[b], pos, invf, cfg.rotary_dim) for b in range(B)])
    k = torch.stack([R.apply_rope(k[b], pos, invf, cfg.rotary_dim) for b in range(B)])
    G = Hq // Hkv
    kr = k.repeat_interleave(G, dim=2)
    vr = v.repeat_interleave(G, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q, kr) / math.sqrt(D)
    mask = torch.ones(S, S, dtype=torch.bool, device=x.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), vr).reshape(B, S, Hq * D)
    if cfg.attn_output_gate:
        gate = qkv[..., (Hq + 2 * Hkv) * D:]
        o = o * torch.sigmoid(gate)
    y = o @ _f(aw.o).t()
    if aw.o_bias is not None:
        y = y + _f(aw.o_bias)
    return y


def deltanet_block(cfg: ModelConfig, dw, x):
    """Gated delta rule, sequential over time (fp32)."""
    B, S, H = x.shape
    Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
    dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
    kd, vd = Hk * dk, Hv * dv
    p = x @ _f(dw.in_qkvz).t()
    qkv, z = p[..., : 2 * kd + vd], p[..., 2 * kd + vd:]
    ba = x @ _f(dw.in_ba).t()
    b, a = ba[..., :Hv], ba[..., Hv:]
    # causal depthwise conv (kernel K) + SiLU over the q/k/v channels
    Kc = dw.conv.shape[1]
    xc = F.pad(qkv.transpose(1, 2), (Kc - 1, 0))                  # [B, C, S+K-1]
    qkv = F.silu(F.conv1d(xc, _f(dw.conv)[:, None, :], groups=qkv.shape[-1])).transpose(1, 2)
    q = qkv[..., :kd].reshape(B, S, Hk, dk)
    k = qkv[..., kd:2 * kd].reshape(B, S, Hk, dk)
    v = qkv[..., 2 * kd:].reshape(B, S, Hv, dv)
    rep = Hv // Hk
    q = F.normalize(q, dim=-1).repeat_interleave(rep, dim=2) / math.sqrt(dk)
    k = F.normalize(k, dim=-1).repeat_interleave(rep, dim=2)
    beta = torch.sigmoid(b)                                        # [B, S, Hv]
    g = -torch.exp(dw.A_log.float()) * F.softplus(a + dw.dt_bias.float())
    state = torch.zeros(B, Hv, dk, dv, device=x.device)
    outs = []
    for t in range(S):
        state = state * torch.exp(g[:, t])[:, :, None, None]
        kv_mem = torch.einsum("bhkv,bhk->bhv", state, k[:, t])
        delta = (v[:, t] - kv_mem) * beta[:, t][:, :, None]
        state = state + torch.einsum("bhk,bhv->bhkv", k[:, t], delta)
        outs.append(torch.einsum("bhkv,bhk->bhv", state, q[:, t]))
    o = torch.stack(outs, dim=1)                                   # [B, S, Hv, dv]
    o = rms(o, _f(dw.norm), cfg.rms_norm_eps) * F.silu(z.reshape(B, S, Hv, dv))
    return o.reshape(B, S, vd) @ _f(dw.out).t()


def mlp_block(cfg: ModelConfig, mw, x):
    if mw.gate_up is not None:
        gu = x @ _f(mw.gate_up).t()
        I = gu.shape[-1] // 2
        return (F.silu(gu[..., :I]) * gu[..., I:]) @ _f(mw.down).t()
    h = x @ _f(mw.up).t() + _f(mw.up_bias)
    return (F.gelu(h, approximate="tanh") @ _f(mw.down).t()) + _f(mw.down_bias)


def moe_block(cfg: ModelConfig, mo, x):
    B, S, H = x.shape
    xt = x.reshape(-1, H)
    logits = xt @ _f(mo.router).t()
    p = torch.softmax(logits, -1)
    w, ids = torch.topk(p, cfg.num_experts_per_tok, dim=-1)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    I = cfg.moe_intermediate_size
    E = mo.e_hi - mo.e_lo
    w13 = _f(mo.w13).view(E, 2 * I, H)
    w2 = _f(mo.w2).view(E, H, I)
    out = torch.zeros_like(xt)
    for e in range(E):
        tok, slot = (ids == e + mo.e_lo).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        gu = xt[tok] @ w13[e].t()
        ye = (F.silu(gu[:, :I]) * gu[:, I:]) @ w2[e].t()
        out.index_add_(0, tok, ye * w[tok, slot][:, None])
    if mo.shared is not None:
        sh = mlp_block(cfg, mo.shared, xt)
        out = out + torch.sigmoid(xt @ _f(mo.shared_gate).t()) * sh
    return out.reshape(B, S, H)


@torch.no_grad()
def forward(cfg: ModelConfig, w: ModelWeights, ids: torch.Tensor, inputs_embeds: torch.Tensor = None) -> torch.Tensor:
    """ids [B, S] -> logits [B, S, V] in fp32."""
    x = inputs_embeds.float() if inputs_embeds is not None else _f(w.embed)[ids]
    B, S, _ = x.shape
    pos = torch.arange(S, device=x.device)
    eps = cfg.rms_norm_eps
    for L in w.layers:
        h = rms(x, _f(L.in_norm), eps)
        if L.kind == "full_attention":
            x = x + attention_block(cfg, L.attn, h, pos)
        else:
            x = x + deltanet_block(cfg, L.delta, h)
        h = rms(x, _f(L.post_norm), eps)
        x = x + (moe_block(cfg, L.moe, h) if L.moe is not None else mlp_block(cfg, L.mlp, h))
    x = rms(x, _f(w.final_norm), eps)
    return x @ _f(w.lm_head).t()


@torch.no_grad()
def greedy_generate(cfg: ModelConfig, w: ModelWeights, ids: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
    """Greedy decode by full recomputation (oracle for token-match tests)."""
    out = ids
    for _ in range(max_new_tokens):
        logits = forward(cfg, w, out)
        nxt = logits[:, -1].argmax(-1, keepdim=True)
        out = torch.cat([out, nxt], dim=1)
    return out[:, ids.shape[1]:]
