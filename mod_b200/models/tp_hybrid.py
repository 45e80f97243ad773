"""Tensor-parallel hybrid decoder (Qwen3-Next family: gated DeltaNet and gated
attention layers, routed experts with a shared expert) with a
sequence-parallel residual stream.

Per layer and rank:

* token mixer: the owners' normed rows are all-gathered into the mixer's
  column-parallel input GEMM (this rank's attention heads, or its DeltaNet key
  / value heads with their conv channels, gates and z rows); the heads run
  locally; the row-parallel output GEMM's partials are reduce-scattered to the
  token owners with the residual add and the post-mixer RMSNorm fused in
  (:mod:`mod_b200.parallel.tp` boundaries);
* MoE: each rank routes the tokens it owns through the expert-parallel
  exchange over the same ranks (E/N experts each, the shared expert on the
  owner), and the output joins the residual in the next boundary, which also
  pushes the next layer's normed rows.

Query heads split evenly; with fewer KV heads than ranks each rank keeps the
one KV head its query heads read (replicated across the ranks of a group).
DeltaNet key and value heads split evenly (the value heads of a key head stay
together).  The reference's hybrid model runs on one device
(``pio/models/qwen3_coder_next/model.py:425-472``).
"""
from __future__ import annotations

from typing import Optional

import torch

from ..config.models import ModelConfig
from ..engine.batch import ForwardBatch
from ..engine.kv_cache import KVCache, StateCache
from ..ops import reference as R
from ..parallel.tp import padded_tokens
from .deltanet import DeltaNetLayer
from .tp_decoder import _prefill_ref
from .weights import AttnWeights, DeltaNetWeights, LayerWeights, MLPWeights, ModelWeights, MoEWeights


def attn_heads(cfg: ModelConfig, rank: int, world: int):
    """(first query head, query heads, first KV head, KV heads) of ``rank``."""
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    assert Hq % world == 0, "query heads must split evenly"
    hq = Hq // world
    if Hkv % world == 0:
        return rank * hq, hq, rank * (Hkv // world), Hkv // world
    group = Hq // Hkv                      # query heads per KV head
    assert world % Hkv == 0 and group % hq == 0, "each rank's query heads must share one KV head"
    return rank * hq, hq, (rank * hq) // group, 1


def _shard_attn(cfg, a: AttnWeights, rank, world) -> AttnWeights:
    assert a.qkv_bias is None and a.o_bias is None, "tensor-parallel attention without biases"
    D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    q0, hq, k0, hk = attn_heads(cfg, rank, world)
    rows = [a.qkv[q0 * D:(q0 + hq) * D],
            a.qkv[(Hq + k0) * D:(Hq + k0 + hk) * D],
            a.qkv[(Hq + Hkv + k0) * D:(Hq + Hkv + k0 + hk) * D]]
    if cfg.attn_output_gate:               # gate rows follow q | k | v
        g0 = (Hq + 2 * Hkv) * D
        rows.append(a.qkv[g0 + q0 * D:g0 + (q0 + hq) * D])
    return AttnWeights(qkv=torch.cat(rows).contiguous(), o=a.o[:, q0 * D:(q0 + hq) * D].contiguous(),
                       q_norm=a.q_norm, k_norm=a.k_norm)


def _shard_delta(cfg, d: DeltaNetWeights, rank, world) -> DeltaNetWeights:
    Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
    dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
    assert Hk % world == 0 and Hv % world == 0, "DeltaNet heads must split evenly"
    hk, hv = Hk // world, Hv // world
    kd, vd = Hk * dk, Hv * dv
    qs, vs = slice(rank * hk * dk, (rank + 1) * hk * dk), slice(rank * hv * dv, (rank + 1) * hv * dv)

    def off(sl, o):
        return slice(sl.start + o, sl.stop + o)

    in_qkvz = torch.cat([d.in_qkvz[qs], d.in_qkvz[off(qs, kd)], d.in_qkvz[off(vs, 2 * kd)],
                         d.in_qkvz[off(vs, 2 * kd + vd)]]).contiguous()
    hs = slice(rank * hv, (rank + 1) * hv)
    in_ba = torch.cat([d.in_ba[hs], d.in_ba[off(hs, Hv)]]).contiguous()
    conv = torch.cat([d.conv[qs], d.conv[off(qs, kd)], d.conv[off(vs, 2 * kd)]]).contiguous()
    return DeltaNetWeights(in_qkvz=in_qkvz, in_ba=in_ba, conv=conv, A_log=d.A_log[hs].contiguous(),
                           dt_bias=d.dt_bias[hs].contiguous(), norm=d.norm, out=d.out[:, vs].contiguous())


def _shard_moe(cfg, m: MoEWeights, rank, world) -> MoEWeights:
    """This rank's experts [r*E/N, (r+1)*E/N); router and shared expert whole."""
    E, I, H = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size
    El = E // world
    lo, hi = rank * El, (rank + 1) * El
    if m.e_hi - m.e_lo == El and m.e_lo == lo:
        return m                           # already this rank's experts
    assert (m.e_lo, m.e_hi) in ((0, E), (0, 0)), "expert shard does not match the rank"
    return MoEWeights(router=m.router, w13=m.w13[lo * 2 * I:hi * 2 * I].contiguous(),
                      w2=m.w2[lo * H:hi * H].contiguous(), shared=m.shared, shared_gate=m.shared_gate,
                      e_lo=lo, e_hi=hi)


def shard_hybrid_weights(cfg: ModelConfig, w: ModelWeights, rank: int, world: int) -> ModelWeights:
    layers = []
    for L in w.layers:
        n = LayerWeights(kind=L.kind, in_norm=L.in_norm, post_norm=L.post_norm)
        if L.attn is not None:
            n.attn = _shard_attn(cfg, L.attn, rank, world)
        if L.delta is not None:
            n.delta = _shard_delta(cfg, L.delta, rank, world)
        if L.moe is not None:
            n.moe = _shard_moe(cfg, L.moe, rank, world)
        if L.mlp is not None:
            I = cfg.intermediate_size
            assert L.mlp.gate_up is not None and I % world == 0
            il = I // world
            g, u = L.mlp.gate_up.split([I, I])
            n.mlp = MLPWeights(gate_up=torch.cat([g[rank * il:(rank + 1) * il], u[rank * il:(rank + 1) * il]])
                               .contiguous(), down=L.mlp.down[:, rank * il:(rank + 1) * il].contiguous())
        layers.append(n)
    return ModelWeights(embed=w.embed, layers=layers, final_norm=w.final_norm, lm_head=w.lm_head)


class TPHybridLM:
    def __init__(self, cfg: ModelConfig, weights: ModelWeights, backend, comm, world: int, moe_impl=None):
        """``weights``: this rank's shard (:func:`shard_hybrid_weights`); ``comm``: the TP boundary
        object (``FusedTP`` / ``NvlsTP`` / ``NcclTP``); ``moe_impl``: the expert-parallel exchange
        over the same ranks (``FusedEPMoE`` / ``NcclEPMoE``)."""
        self.cfg, self.w, self.be, self.comm, self.world = cfg, weights, backend, comm, world
        self.moe_impl = moe_impl
        r = comm.rank
        _, self.Hq, _, self.Hkv = attn_heads(cfg, r, world) if cfg.num_attention_heads else (0, 0, 0, 0)
        self.hk = cfg.linear_num_key_heads // world if cfg.linear_num_key_heads else 0
        self.hv = cfg.linear_num_value_heads // world if cfg.linear_num_value_heads else 0
        self.device = weights.embed.device
        self.inv_freq = R.inv_freq(cfg.rotary_dim, cfg.rope_theta, device=self.device)
        self.delta = {i: DeltaNetLayer(cfg, L.delta, num_k_heads=self.hk, num_v_heads=self.hv)
                      for i, L in enumerate(weights.layers) if L.delta is not None}
        # the mixer's column-parallel input weights, one GEMM per layer, padded with zero rows to a
        # multiple of 128 outputs (the decode GEMMs' tile; the extra columns are never read)
        self.in_w = []
        for L in weights.layers:
            w = L.attn.qkv if L.attn is not None else torch.cat([L.delta.in_qkvz, L.delta.in_ba])
            pad = -w.shape[0] % 128
            if pad:
                w = torch.cat([w, w.new_zeros(pad, w.shape[1])])
            self.in_w.append(w.contiguous())
        self.layer_source = None

    def state_cache(self, max_seqs: int, device) -> StateCache:
        return StateCache(self.cfg, max_seqs, device, num_v_heads=self.hv, num_k_heads=self.hk)

    def _attention(self, i, L, qkv, fb: ForwardBatch, kv: KVCache):
        cfg, be = self.cfg, self.be
        T, D, hq, hkv = qkv.shape[0], cfg.head_dim, self.Hq, self.Hkv
        kc, vc = kv.layer(i)
        q = torch.empty(T, hq, D, dtype=qkv.dtype, device=qkv.device)
        be.rope_qknorm(qkv, L.attn.q_norm, L.attn.k_norm, fb.positions, self.inv_freq, fb.slot_mapping, q, kc, vc,
                       hq, hkv, D, cfg.rotary_dim, cfg.rms_norm_eps)
        if fb.is_decode:
            o = be.attn_decode(q, kc, vc, fb.block_tables, fb.ctx_lens, fb.attn_splits)
        else:
            o = be.attn_prefill_paged(q, kc, vc, fb) if hasattr(be, "attn_prefill_paged") else None
            if o is None:
                o = _prefill_ref(q, kc, vc, fb)
        o = o.reshape(T, hq * D)
        if cfg.attn_output_gate:
            gate = qkv[:, (hq + 2 * hkv) * D:(2 * hq + 2 * hkv) * D]
            o = (o.float() * torch.sigmoid(gate.float())).to(qkv.dtype)
        return o

    def _deltanet(self, i, y, fb: ForwardBatch, states: StateCache):
        layer = self.delta[i]
        kd, vd = self.hk * self.cfg.linear_key_head_dim, self.hv * self.cfg.linear_value_head_dim
        conv, ssm = states.layer(i)
        b0 = 2 * kd + 2 * vd
        return layer.core(self.be, y[:, :2 * kd + vd], y[:, 2 * kd + vd:b0], y[:, b0:b0 + 2 * self.hv],
                          conv, ssm, fb)

    def forward(self, fb: ForwardBatch, kv: Optional[KVCache], states: Optional[StateCache] = None) -> torch.Tensor:
        cfg, be, comm = self.cfg, self.be, self.comm
        eps, H = cfg.rms_norm_eps, cfg.hidden_size
        T = fb.input_ids.shape[0]
        Tp = padded_tokens(T, self.world)
        pr = Tp // self.world
        r = comm.rank
        ids = fb.input_ids
        if Tp != T:
            ids = torch.cat([ids, ids.new_zeros(Tp - T)])
        h = be.embed(ids[r * pr:(r + 1) * pr].contiguous(), self.w.embed)   # residual shard [pr, H]
        layers = self.w.layers
        comm.publish(h, layers[0].in_norm, eps, partials=False)
        for i, L in enumerate(layers):
            y = comm.ag_gemm(self.in_w[i], Tp)[:T]
            if L.attn is not None:
                o, out_w = self._attention(i, L, y, fb, kv), L.attn.o
            else:
                o, out_w = self._deltanet(i, y, fb, states), L.delta.out
            o2 = torch.zeros(Tp, o.shape[1], dtype=o.dtype, device=o.device)
            o2[:T] = o
            comm.gemm_rs(o2, out_w)
            nxt = layers[i + 1].in_norm if i + 1 < len(layers) else self.w.final_norm
            if L.moe is not None:
                xn = torch.empty(pr, H, dtype=h.dtype, device=h.device)
                comm.publish(h, L.post_norm, eps, partials=True, local_out=xn)
                if self.moe_impl is not None:
                    m = self.moe_impl(xn, L.moe)
                else:
                    m = be.moe(xn, L.moe, cfg.num_experts_per_tok, cfg.norm_topk_prob, cfg.moe_intermediate_size)
                comm.publish(h, nxt, eps, partials=False, x_add=m.to(h.dtype))
            else:
                comm.publish(h, L.post_norm, eps, partials=True)
                hmid = comm.ag_gemm(L.mlp.gate_up, Tp, swiglu=True)
                comm.gemm_rs(hmid, L.mlp.down)
                comm.publish(h, nxt, eps, partials=True)
        return comm.gather_rows(fb.logits_idx, Tp)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.be.linear(h, self.w.lm_head)

    def sample_greedy(self, h: torch.Tensor) -> torch.Tensor:
        return self.be.argmax(self.logits(h))
