"""Tensor-parallel dense decoder (Qwen3 dense family) with a sequence-parallel
residual stream; the collectives are :mod:`mod_b200.parallel.tp` boundaries.

Per rank: query heads [r*Hq/N, ...), KV heads [r*Hkv/N, ...), an I/N slice of
the MLP, the replicated embedding / norms / LM head.  The decode step is
CUDA-graph capturable with the fused boundaries (no host work inside).
"""
from __future__ import annotations

from dataclasses import replace
from typing import Optional

import torch

from ..config.models import ModelConfig
from ..engine.batch import ForwardBatch
from ..engine.kv_cache import KVCache
from ..ops import reference as R
from ..parallel.tp import padded_tokens
from .weights import AttnWeights, LayerWeights, MLPWeights, ModelWeights


def shard_weights(cfg: ModelConfig, w: ModelWeights, rank: int, world: int) -> ModelWeights:
    """Column-parallel QKV / gate-up, row-parallel o / down; the rest replicated."""
    Hq, Hkv, D, I = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.intermediate_size
    assert Hq % world == 0 and Hkv % world == 0 and I % world == 0, "heads and MLP must split evenly"
    hq, hk, il = Hq // world, Hkv // world, I // world
    layers = []
    for L in w.layers:
        q, k, v = L.attn.qkv.split([Hq * D, Hkv * D, Hkv * D])
        qkv = torch.cat([q[rank * hq * D:(rank + 1) * hq * D], k[rank * hk * D:(rank + 1) * hk * D],
                         v[rank * hk * D:(rank + 1) * hk * D]]).contiguous()
        o = L.attn.o[:, rank * hq * D:(rank + 1) * hq * D].contiguous()
        g, u = L.mlp.gate_up.split([I, I])
        gu = torch.cat([g[rank * il:(rank + 1) * il], u[rank * il:(rank + 1) * il]]).contiguous()
        down = L.mlp.down[:, rank * il:(rank + 1) * il].contiguous()
        layers.append(LayerWeights(kind=L.kind, in_norm=L.in_norm, post_norm=L.post_norm,
                                   attn=AttnWeights(qkv=qkv, o=o, q_norm=L.attn.q_norm, k_norm=L.attn.k_norm),
                                   mlp=MLPWeights(gate_up=gu, down=down)))
    return ModelWeights(embed=w.embed, layers=layers, final_norm=w.final_norm, lm_head=w.lm_head)


class TPDecoderLM:
    def __init__(self, cfg: ModelConfig, weights: ModelWeights, backend, comm, world: int):
        """``weights`` is this rank's shard (see :func:`shard_weights`); ``comm`` is a
        ``FusedTP`` or ``NcclTP`` boundary implementation."""
        assert not cfg.is_moe and cfg.hidden_act == "silu" and not cfg.attention_bias
        self.cfg, self.w, self.be, self.comm, self.world = cfg, weights, backend, comm, world
        self.Hq = cfg.num_attention_heads // world
        self.Hkv = cfg.num_key_value_heads // world
        self.device = weights.embed.device
        self.inv_freq = R.inv_freq(cfg.rotary_dim, cfg.rope_theta, device=self.device)
        self.layer_source = None

    def forward(self, fb: ForwardBatch, kv: KVCache, states=None) -> torch.Tensor:
        cfg, be, comm = self.cfg, self.be, self.comm
        eps, H, D = cfg.rms_norm_eps, cfg.hidden_size, cfg.head_dim
        T = fb.input_ids.shape[0]
        Tp = padded_tokens(T, self.world)
        pr = Tp // self.world
        r = comm.rank
        ids = fb.input_ids
        if Tp != T:
            ids = torch.cat([ids, ids.new_zeros(Tp - T)])
        if fb.inputs_embeds is not None:  # this rank's shard rows, prepared by the caller (image tokens)
            h = fb.inputs_embeds.contiguous().clone()
        else:
            h = be.embed(ids[r * pr:(r + 1) * pr].contiguous(), self.w.embed)   # residual shard [pr, H]
        layers = self.w.layers
        comm.publish(h, layers[0].in_norm, eps, partials=False)
        for i, L in enumerate(layers):
            aw = L.attn
            kc, vc = kv.layer(i)
            q = torch.empty(T, self.Hq, D, dtype=h.dtype, device=h.device)
            fused = hasattr(comm, "ag_qkv_rope") and comm.ag_qkv_rope(
                aw.qkv, T, aw.q_norm, aw.k_norm, fb.positions, self.inv_freq, fb.slot_mapping, q, kc, vc, self.Hq,
                self.Hkv, D, cfg.rotary_dim, eps)
            if not fused:
                qkv = comm.ag_gemm(aw.qkv, Tp)[:T]
                be.rope_qknorm(qkv, aw.q_norm, aw.k_norm, fb.positions, self.inv_freq, fb.slot_mapping, q, kc, vc,
                               self.Hq, self.Hkv, D, cfg.rotary_dim, eps)
            if fb.is_decode:
                o = be.attn_decode(q, kc, vc, fb.block_tables, fb.ctx_lens, fb.attn_splits)
            else:
                o = be.attn_prefill_paged(q, kc, vc, fb) if hasattr(be, "attn_prefill_paged") else None
                if o is None:
                    o = _prefill_ref(q, kc, vc, fb)
            o2 = torch.zeros(Tp, self.Hq * D, dtype=o.dtype, device=o.device)
            o2[:T] = o.reshape(T, -1)
            comm.gemm_rs(o2, aw.o)
            comm.publish(h, L.post_norm, eps, partials=True)
            hmid = comm.ag_gemm(L.mlp.gate_up, Tp, swiglu=True)
            comm.gemm_rs(hmid, L.mlp.down)
            nxt = layers[i + 1].in_norm if i + 1 < len(layers) else self.w.final_norm
            comm.publish(h, nxt, eps, partials=True)
        return comm.gather_rows(fb.logits_idx, Tp)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.be.linear(h, self.w.lm_head)

    def sample_greedy(self, h: torch.Tensor) -> torch.Tensor:
        """Greedy tokens.  With the fused boundaries the LM head is vocabulary-parallel: each rank
        multiplies its 1/N row slice of the (replicated) head, takes the best logit of its slice
        and the ranks exchange one (value, index) pair per token row over NVLink, so a step reads
        1/N of the head instead of all of it (``pio/plugins/cuda/c_src/tensor_ops_cuda.cu:782-788``
        is the reference's full-vocabulary argmax launch)."""
        V = self.w.lm_head.shape[0]
        if (not hasattr(self.comm, "argmax_exchange") or V % self.world or not hasattr(self.be, "N")
                or not isinstance(self.w.lm_head, torch.Tensor)):
            return self.be.argmax(self.logits(h))
        Vl = V // self.world
        r = self.comm.rank
        local = self.be.linear(h, self.w.lm_head[r * Vl:(r + 1) * Vl])   # a row slice: a contiguous view
        vals = torch.empty(h.shape[0], dtype=torch.float32, device=h.device)
        idxs = self.be.N.argmax(local, out_val=vals, index_offset=r * Vl)
        return self.comm.argmax_exchange(vals, idxs)


def _prefill_ref(q, kc, vc, fb):
    o = torch.empty_like(q)
    start = 0
    for b, ql in enumerate(fb.query_lens):
        n = fb.ctx_lens_host[b]
        k = R.gather_kv(kc, fb.block_tables[b], n)
        v = R.gather_v(vc, fb.block_tables[b], n)
        qb = q[start:start + ql]
        mask = torch.arange(n, device=q.device)[None, :] <= (n - ql + torch.arange(ql, device=q.device))[:, None]
        ob = torch.nn.functional.scaled_dot_product_attention(qb.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                              v.transpose(0, 1)[None], attn_mask=mask[None, None],
                                                              enable_gqa=True)
        o[start:start + ql] = ob[0].transpose(0, 1)
        start += ql
    return o
