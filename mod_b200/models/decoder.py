"""Engine-side decoder LM: Qwen3 dense / Qwen3 MoE / Qwen3-Next hybrid / GLM.

One class runs every family; the per-layer kind (full attention or gated
DeltaNet) and the MLP kind (SwiGLU, GELU, routed experts) come from the
config.  The residual stream follows the fused "add + norm" pattern: each
block returns its output and the next RMSNorm adds it to the residual in the
same kernel.

Reference model code: ``pio/models/qwen3_0_6b/architecture.py:68-221`` (dense),
``pio/models/qwen3_coder_30b/model.py:291-358`` (MoE),
``pio/models/qwen3_coder_next/model.py:51-472`` (hybrid),
``pio/models/glm_4_7_flash/model.py:186-306`` (GLM).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from ..config.models import ModelConfig
from ..engine.batch import ForwardBatch
from ..engine.kv_cache import KVCache, StateCache
from ..ops import reference as R
from .deltanet import DeltaNetLayer
from .weights import ModelWeights
from ..utils import tracing


class DecoderLM:
    def __init__(self, cfg: ModelConfig, weights: ModelWeights, backend, moe_impl=None, tp=None):
        """``moe_impl`` (optional) replaces the local MoE block, e.g. by the
        expert-parallel dispatch/combine; ``tp`` holds tensor-parallel head
        counts when attention is sharded."""
        cfg.validate()
        self.cfg, self.w, self.be = cfg, weights, backend
        self.moe_impl = moe_impl
        dev = weights.embed.device
        self.Hq = tp["heads"] if tp else cfg.num_attention_heads
        self.Hkv = tp["kv_heads"] if tp else cfg.num_key_value_heads
        self.inv_freq = R.inv_freq(cfg.rotary_dim, cfg.rope_theta, device=dev)
        self.delta = {i: DeltaNetLayer(cfg, L.delta) for i, L in enumerate(weights.layers) if L.delta is not None}
        self.device = dev
        self.layer_source = None  # optional i -> LayerWeights (weight streaming)

    # ------------------------------------------------------------------ blocks
    def _attention(self, i, L, x, fb: ForwardBatch, kv: KVCache):
        cfg, be, aw = self.cfg, self.be, L.attn
        T = x.shape[0]
        Hq, Hkv, D = self.Hq, self.Hkv, cfg.head_dim
        kc, vc = kv.layer(i)
        q = torch.empty(T, Hq, D, dtype=x.dtype, device=x.device)
        fused = (aw.qkv_bias is None and not cfg.attn_output_gate and hasattr(be, "qkv_rope")
                 and be.qkv_rope(x, aw.qkv, aw.q_norm, aw.k_norm, fb.positions, self.inv_freq, fb.slot_mapping, q, kc,
                                 vc, Hq, Hkv, D, cfg.rotary_dim, cfg.rms_norm_eps))
        if not fused:
            qkv = be.linear(x, aw.qkv, bias=aw.qkv_bias)
            be.rope_qknorm(qkv, aw.q_norm, aw.k_norm, fb.positions, self.inv_freq, fb.slot_mapping, q, kc, vc, Hq,
                           Hkv, D, cfg.rotary_dim, cfg.rms_norm_eps)
        if hasattr(be, "attn_paged"):
            o = be.attn_paged(q, kc, vc, fb)
        elif fb.is_decode:
            o = be.attn_decode(q, kc, vc, fb.block_tables, fb.ctx_lens, fb.attn_splits)
        elif hasattr(be, "attn_prefill_paged") and (o := be.attn_prefill_paged(q, kc, vc, fb)) is not None:
            pass
        else:
            o = torch.empty_like(q)
            start = 0
            for b, ql in enumerate(fb.query_lens):
                n = fb.ctx_lens_host[b]
                k = R.gather_kv(kc, fb.block_tables[b], n)
                v = R.gather_v(vc, fb.block_tables[b], n)
                qb = q[start:start + ql]
                if ql == n:
                    o[start:start + ql] = be.attn_prefill(qb, k, v)
                else:  # prefix already cached: causal with an offset
                    mask = torch.arange(n, device=x.device)[None, :] <= (n - ql + torch.arange(ql, device=x.device))[:, None]
                    ob = F.scaled_dot_product_attention(qb.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                        v.transpose(0, 1)[None], attn_mask=mask[None, None],
                                                        enable_gqa=True)
                    o[start:start + ql] = ob[0].transpose(0, 1)
                start += ql
        o = o.reshape(T, Hq * D)
        if cfg.attn_output_gate:
            gate = qkv[:, (Hq + 2 * Hkv) * D:(2 * Hq + 2 * Hkv) * D]
            o = (o.float() * torch.sigmoid(gate.float())).to(x.dtype)
        return be.linear(o, aw.o, bias=aw.o_bias)

    def _deltanet(self, i, x, fb: ForwardBatch, states: StateCache):
        layer = self.delta[i]
        conv, ssm = states.layer(i)
        if layer._native(self.be, x):
            if fb.is_decode:
                return layer.decode_native(self.be, x, conv, ssm, fb.state_slots)
            return layer.prefill_native(self.be, x, conv, ssm, fb.state_slots, fb.query_lens)
        if fb.is_decode:
            return layer.decode(self.be, x, conv, ssm, fb.state_slots)
        outs = []
        start = 0
        slots = fb.state_slots.tolist()
        for b, ql in enumerate(fb.query_lens):
            outs.append(layer.prefill(self.be, x[start:start + ql], conv, ssm, slots[b]))
            start += ql
        return torch.cat(outs, 0)

    def _mlp(self, L, x):
        cfg, be = self.cfg, self.be
        if L.moe is not None:
            if self.moe_impl is not None:
                if getattr(self.moe_impl, "supports_defer", False):
                    return self.moe_impl(x, L.moe, defer=True)
                return self.moe_impl(x, L.moe)
            return be.moe(x, L.moe, cfg.num_experts_per_tok, cfg.norm_topk_prob, cfg.moe_intermediate_size)
        m = L.mlp
        if m.gate_up is not None:
            return be.swiglu_mlp(x, m.gate_up, m.down)
        h = be.linear(x, m.up, bias=m.up_bias)
        h = F.gelu(h.float(), approximate="tanh").to(x.dtype)
        return be.linear(h, m.down, bias=m.down_bias)

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, kv: Optional[KVCache], states: Optional[StateCache] = None) -> torch.Tensor:
        """Returns the final-normed hidden rows selected by ``fb.logits_idx`` [B, H]."""
        cfg, be, w = self.cfg, self.be, self.w
        eps = cfg.rms_norm_eps
        hidden = fb.inputs_embeds if fb.inputs_embeds is not None else be.embed(fb.input_ids, w.embed)
        residual = None
        nv = tracing.nvtx_enabled()
        for i, L in enumerate(w.layers):
            if self.layer_source is not None:
                L = self.layer_source(i)
            if nv:
                torch.cuda.nvtx.range_push(f"layer{i}:{L.kind}")
            if residual is None:
                residual = hidden.clone()
                x = be.rmsnorm(hidden, L.in_norm, eps)
            else:
                x = self._add_norm(hidden, L.in_norm, eps, residual)
            if L.kind == "full_attention":
                hidden = self._attention(i, L, x, fb, kv)
            else:
                hidden = self._deltanet(i, x, fb, states)
            x = be.rmsnorm(hidden, L.post_norm, eps, residual=residual)
            hidden = self._mlp(L, x)
            if nv:
                torch.cuda.nvtx.range_pop()
        x = self._add_norm(hidden, w.final_norm, eps, residual)
        return x.index_select(0, fb.logits_idx)

    def _add_norm(self, hidden, w, eps, residual):
        """residual += hidden; returns rmsnorm(residual) * w.  An expert-parallel
        MoE output still in flight finishes its combine inside this step."""
        if hasattr(hidden, "add_norm"):
            return hidden.add_norm(residual, w, eps)
        return self.be.rmsnorm(hidden, w, eps, residual=residual)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.be.linear(h, self.w.lm_head)

    def sample_greedy(self, h: torch.Tensor) -> torch.Tensor:
        return self.be.argmax(self.logits(h))
