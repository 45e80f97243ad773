"""Checkpoint I/O: HF safetensors layout -> fused :class:`ModelWeights`.

Files are read through the C++ mmap reader (``mod_b200._cpu.SafeTensorsFile``):
a tensor is a zero-copy view of the mapping until it is cast and moved to the
device, and an expert-parallel rank only touches its own experts.  Single
files and ``model.safetensors.index.json`` shards are both accepted
(``pio/common/custom_components/model_loader.py:95-123`` does the same with a
``strstr`` header scan and F16-decodes BF16 data).

Name mapping (HF Qwen3 / Qwen3-MoE / Qwen3-Next / GLM-style):
  q/k/v_proj (+ attention gate rows of Qwen3-Next q_proj) -> attn.qkv
  gate/up_proj -> mlp.gate_up;  experts.{e}.gate/up -> moe.w13;  experts.{e}.down -> moe.w2
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterable, Optional, Tuple

import torch

from ..config.models import ModelConfig
from .upload import StagedUploader
from ..models.weights import (AttnWeights, DeltaNetWeights, LayerWeights, MLPWeights, ModelWeights, MoEWeights)


def _cpu():
    import importlib

    return importlib.import_module("mod_b200._cpu")


class CheckpointReader:
    """Name -> tensor over one file or an index of shards."""

    def __init__(self, path: str):
        C = _cpu()
        self.files: Dict[str, object] = {}
        self.where: Dict[str, str] = {}
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as f:
                    wm = json.load(f)["weight_map"]
                for name, fn in wm.items():
                    self.where[name] = os.path.join(path, fn)
            else:
                fn = os.path.join(path, "model.safetensors")
                path = fn
        if not self.where:
            f = C.SafeTensorsFile(path)
            self.files[path] = f
            for k in f.keys():
                self.where[k] = path

    def _file(self, name: str):
        fn = self.where[name]
        if fn not in self.files:
            self.files[fn] = _cpu().SafeTensorsFile(fn)
        return self.files[fn]

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def keys(self) -> Iterable[str]:
        return self.where.keys()

    def get(self, name: str) -> torch.Tensor:
        return self._file(name).get(name)

    def get_slice(self, name: str, dim: int, rank: int, world: int) -> torch.Tensor:
        return self._file(name).get_slice(name, dim, rank, world)


def load_hf(cfg: ModelConfig, path: str, device="cuda", dtype=torch.bfloat16,
            expert_range: Optional[Tuple[int, int]] = None,
            tp: Optional[Tuple[int, int]] = None) -> ModelWeights:
    """HF checkpoint -> fused weights on ``device``.

    ``expert_range=(lo, hi)``: an expert-parallel rank reads experts [lo, hi) only.
    ``tp=(rank, world)``: a tensor-parallel rank of the dense decoder reads its
    own slice of every sharded projection straight from the mapping
    (column-parallel q/k/v and gate/up rows, row-parallel o and down columns;
    embedding, norms and LM head replicated), the same layout as
    ``models.tp_decoder.shard_weights`` of the full weights, without ever
    materialising the full projection (``pio/common/custom_components/
    model_loader.py:77-123`` loads whole tensors only).
    """
    r = CheckpointReader(path)
    trank, tworld = tp or (0, 1)
    if tworld > 1:
        assert not cfg.is_moe and not cfg.attn_output_gate and all(
            cfg.layer_type(i) == "full_attention" for i in range(cfg.num_hidden_layers)), \
            "tensor-parallel loading covers the dense attention decoder"

    # CUDA targets go through two pinned staging buffers, so mapping reads overlap the copies
    up = StagedUploader(device) if torch.device(device).type == "cuda" else None

    def put(x, dt=dtype):
        return up.upload(x, dt) if up is not None else x.to(device=device, dtype=dt)

    def t(name):
        return put(r.get(name))

    def sl(name, dim):
        """This TP rank's 1/world of ``name`` along ``dim`` (the whole tensor at world 1)."""
        return r.get_slice(name, dim, trank, tworld) if tworld > 1 else r.get(name)

    def opt(name):
        return t(name) if name in r else None

    H, D = cfg.hidden_size, cfg.head_dim
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        kind = cfg.layer_type(i)
        L = LayerWeights(kind=kind, in_norm=t(p + "input_layernorm.weight"),
                         post_norm=t(p + "post_attention_layernorm.weight"))
        if kind == "full_attention":
            q = sl(p + "self_attn.q_proj.weight", 0)
            gate = None
            if cfg.attn_output_gate:  # q_proj rows are [q_h, gate_h] per head
                qg = q.view(Hq, 2 * D, H)
                q, gate = qg[:, :D].reshape(Hq * D, H), qg[:, D:].reshape(Hq * D, H)
            parts = [q, sl(p + "self_attn.k_proj.weight", 0), sl(p + "self_attn.v_proj.weight", 0)]
            if gate is not None:
                parts.append(gate)
            qkv = put(torch.cat([x.to(dtype) for x in parts], 0))
            bias = None
            if p + "self_attn.q_proj.bias" in r:
                bias = put(torch.cat([sl(p + f"self_attn.{n}_proj.bias", 0).to(dtype) for n in "qkv"], 0))
            L.attn = AttnWeights(qkv=qkv, o=put(sl(p + "self_attn.o_proj.weight", 1)), q_norm=opt(p + "self_attn.q_norm.weight"),
                                 k_norm=opt(p + "self_attn.k_norm.weight"), qkv_bias=bias,
                                 o_bias=opt(p + "self_attn.o_proj.bias"))
            assert tworld == 1 or L.attn.o_bias is None, "a row-parallel o_proj bias would be summed world times"
        else:
            la = p + "linear_attn."
            Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
            dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
            rep = Hv // Hk
            w = r.get(la + "in_proj_qkvz.weight").view(Hk, 2 * dk + 2 * rep * dv, H)
            qkvz = torch.cat([w[:, :dk].reshape(-1, H), w[:, dk:2 * dk].reshape(-1, H),
                              w[:, 2 * dk:2 * dk + rep * dv].reshape(-1, H), w[:, 2 * dk + rep * dv:].reshape(-1, H)], 0)
            ba = r.get(la + "in_proj_ba.weight").view(Hk, 2 * rep, H)
            ba = torch.cat([ba[:, :rep].reshape(-1, H), ba[:, rep:].reshape(-1, H)], 0)
            L.delta = DeltaNetWeights(in_qkvz=put(qkvz), in_ba=put(ba),
                                      conv=put(r.get(la + "conv1d.weight").reshape(-1, cfg.linear_conv_kernel_dim)),
                                      A_log=put(r.get(la + "A_log"), torch.float32),
                                      dt_bias=put(r.get(la + "dt_bias"), torch.float32),
                                      norm=t(la + "norm.weight"), out=t(la + "out_proj.weight"))
        if cfg.is_moe:
            E = cfg.num_experts
            lo, hi = expert_range or (0, E)
            m = p + "mlp."
            w13 = torch.cat([torch.cat([r.get(m + f"experts.{e}.gate_proj.weight"), r.get(m + f"experts.{e}.up_proj.weight")], 0)
                             .to(dtype) for e in range(lo, hi)], 0)
            w13 = put(w13)
            w2 = put(torch.cat([r.get(m + f"experts.{e}.down_proj.weight").to(dtype) for e in range(lo, hi)], 0))
            mo = MoEWeights(router=t(m + "gate.weight"), w13=w13, w2=w2, e_lo=lo, e_hi=hi)
            if m + "shared_expert.gate_proj.weight" in r:
                mo.shared = MLPWeights(gate_up=torch.cat([t(m + "shared_expert.gate_proj.weight"),
                                                          t(m + "shared_expert.up_proj.weight")], 0),
                                       down=t(m + "shared_expert.down_proj.weight"))
                mo.shared_gate = t(m + "shared_expert_gate.weight")
            L.moe = mo
        else:
            m = p + "mlp."
            if m + "gate_proj.weight" in r:
                L.mlp = MLPWeights(gate_up=put(torch.cat([sl(m + "gate_proj.weight", 0).to(dtype),
                                                          sl(m + "up_proj.weight", 0).to(dtype)], 0)),
                                   down=put(sl(m + "down_proj.weight", 1)))
            else:
                assert tworld == 1, "tensor-parallel loading covers the gated (SwiGLU) MLP"
                L.mlp = MLPWeights(up=t(m + "up_proj.weight"), down=t(m + "down_proj.weight"),
                                   up_bias=opt(m + "up_proj.bias"), down_bias=opt(m + "down_proj.bias"))
        layers.append(L)
    embed = t("model.embed_tokens.weight")
    lm = embed if cfg.tie_word_embeddings or "lm_head.weight" not in r else t("lm_head.weight")
    out = ModelWeights(embed=embed, layers=layers, final_norm=t("model.norm.weight"), lm_head=lm)
    if up is not None:
        up.finish()   # the staging buffers are released only after their last copy
    return out


def save_weights(w: ModelWeights, path: str, cfg: Optional[ModelConfig] = None) -> None:
    """Writes the fused weights (our own layout) as one safetensors file."""
    tensors = {name: t.detach().cpu().contiguous() for name, t in w.tensors()}
    meta = {"format": "mod_b200-fused"}
    if cfg is not None:
        meta["config"] = json.dumps(cfg.to_dict())
    from .safetensors import save_file

    save_file(path, tensors, meta)


def load_weights(path: str, cfg: ModelConfig, device="cuda", dtype=None) -> ModelWeights:
    """Reads a file written by :func:`save_weights` into a structure matching ``cfg``."""
    f = _cpu().SafeTensorsFile(path)
    w = _skeleton(cfg)
    for name in f.keys():
        t = f.get(name)
        if dtype is not None and t.is_floating_point() and not name.endswith(("A_log", "dt_bias")):
            t = t.to(dtype)
        _assign(w, name, t.to(device=device))
    if cfg.tie_word_embeddings:
        w.lm_head = w.embed
    return w


def _skeleton(cfg: ModelConfig) -> ModelWeights:
    layers = []
    for i in range(cfg.num_hidden_layers):
        kind = cfg.layer_type(i)
        L = LayerWeights(kind=kind, in_norm=None, post_norm=None)
        if kind == "full_attention":
            L.attn = AttnWeights(qkv=None, o=None)
        else:
            L.delta = DeltaNetWeights(None, None, None, None, None, None, None)
        if cfg.is_moe:
            L.moe = MoEWeights(router=None, w13=None, w2=None, e_lo=0, e_hi=cfg.num_experts)
            if cfg.shared_expert_intermediate_size:
                L.moe.shared = MLPWeights()
        else:
            L.mlp = MLPWeights()
        layers.append(L)
    return ModelWeights(embed=None, layers=layers, final_norm=None, lm_head=None)


def _assign(w: ModelWeights, name: str, t: torch.Tensor) -> None:
    parts = name.split(".")
    if parts[0] in ("embed", "final_norm", "lm_head"):
        setattr(w, parts[0], t)
        return
    L = w.layers[int(parts[1])]
    if len(parts) == 3:
        setattr(L, parts[2], t)
        return
    obj = getattr(L, parts[2])
    for p in parts[3:-1]:
        obj = getattr(obj, p)
    setattr(obj, parts[-1], t)
