"""Placement planner: parallel degrees and per-GPU memory for a model on N GPUs.

The reference places layers round-robin over whatever devices it finds and
migrates them between CPU and GPU (``src/inference_pio/core/model_loader.py:34-56``,
``src/inference_pio/common/managers/hybrid_scheduler.py:40-94``).  On one B200
box the ranks are identical, so the plan is arithmetic over the model's shape:

* weight bytes per tensor group (embedding / LM head, attention, DeltaNet,
  dense MLP, routed experts, shared expert), computed from the config without
  allocating anything;
* MoE models: expert parallelism over all N GPUs with data-parallel attention
  (each rank holds E/N experts and a full copy of the rest); dense models:
  tensor parallelism at the largest degree that divides the heads, KV heads and
  MLP width and is <= N, with data-parallel replicas over the rest;
* when a GPU's share still does not fit, pipeline stages over more GPUs, and
  with no GPUs left, streaming the remaining layers from pinned host memory
  (the hybrid scheduler);
* KV-cache room left per GPU and the number of 16-token blocks it holds.
"""
from dataclasses import asdict, dataclass, field
from typing import Dict, List

GIB = 1 << 30


@dataclass
class WeightBytes:
    embed: int = 0
    lm_head: int = 0
    attention: int = 0      # all full-attention layers
    deltanet: int = 0       # all linear-attention layers
    mlp: int = 0            # dense MLPs
    experts: int = 0        # routed experts (all of them)
    shared: int = 0         # shared experts + routers + norms

    @property
    def total(self) -> int:
        return self.embed + self.lm_head + self.attention + self.deltanet + self.mlp + self.experts + self.shared


@dataclass
class Plan:
    n_gpus: int
    tp: int = 1
    ep: int = 1
    pp: int = 1
    dp: int = 1
    layers_per_stage: List[int] = field(default_factory=list)
    offload_layers: int = 0
    weight_bytes_per_gpu: int = 0
    kv_bytes_per_gpu: int = 0
    kv_blocks_per_gpu: int = 0
    kv_tokens_per_gpu: int = 0
    fits: bool = True
    notes: List[str] = field(default_factory=list)

    def as_dict(self) -> Dict:
        return asdict(self)


def weight_bytes(cfg, bytes_per_param: float = 2.0, int8_projections: bool = False) -> WeightBytes:
    """Bytes of every tensor group; ``int8_projections`` counts projection matrices at 1 byte (+ fp32 scales)."""
    H, b = cfg.hidden_size, bytes_per_param
    pb = 1.0 if int8_projections else b

    def proj(rows, cols):
        return int(rows * cols * pb + (rows * 4 if int8_projections else 0))

    w = WeightBytes()
    w.embed = int(cfg.vocab_size * H * b)
    w.lm_head = 0 if cfg.tie_word_embeddings else int(cfg.vocab_size * H * b)
    for i in range(cfg.num_hidden_layers):
        w.shared += int(2 * H * b)   # norms
        if cfg.layer_type(i) == "full_attention":
            rows = cfg.q_size * (2 if cfg.attn_output_gate else 1) + 2 * cfg.kv_size
            w.attention += proj(rows, H) + proj(H, cfg.q_size)
        else:
            kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
            vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
            w.deltanet += proj(2 * kd + 2 * vd, H) + proj(2 * cfg.linear_num_value_heads, H) + proj(H, vd)
        if cfg.is_moe:
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            w.experts += E * (proj(2 * I, H) + proj(H, I))
            w.shared += int(E * H * b)   # router
            S = cfg.shared_expert_intermediate_size
            if S:
                w.shared += proj(2 * S, H) + proj(H, S) + int(H * b)
        else:
            I = cfg.intermediate_size
            w.mlp += proj(2 * I, H) + proj(H, I) if cfg.hidden_act == "silu" else proj(I, H) + proj(H, I)
    return w


def kv_bytes_per_token(cfg, kv_heads_per_gpu: int, bytes_per_elem: int = 2) -> int:
    n_attn = sum(1 for i in range(cfg.num_hidden_layers) if cfg.layer_type(i) == "full_attention")
    return n_attn * 2 * kv_heads_per_gpu * cfg.head_dim * bytes_per_elem


def _tp_degree(cfg, n: int) -> int:
    t = 1
    for d in range(1, n + 1):
        if n % d == 0 and cfg.num_attention_heads % d == 0 and cfg.num_key_value_heads % d == 0 \
                and cfg.intermediate_size % d == 0:
            t = d
    return t


def _tp_degree_heads(cfg, n: int) -> int:
    """Largest tensor-parallel degree dividing ``n`` whose head split the hybrid / MoE decoder
    supports: query heads split evenly, KV heads split evenly or each rank's query heads share
    one KV head, DeltaNet key and value heads split evenly."""
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    t = 1
    for d in range(1, n + 1):
        if n % d or Hq % d:
            continue
        kv_ok = Hkv % d == 0 or (d % Hkv == 0 and (Hq // Hkv) % (Hq // d) == 0)
        lin_ok = all(h % d == 0 for h in (cfg.linear_num_key_heads, cfg.linear_num_value_heads) if h)
        if kv_ok and lin_ok:
            t = d
    return t


def plan(cfg, n_gpus: int, hbm_bytes: int = 180 * 10**9, reserve_bytes: int = 6 * GIB,
         workspace_bytes: int = 2 * GIB, block_size: int = 16, int8: bool = False, attn: str = "dp") -> Plan:
    """Placement of ``cfg`` on ``n_gpus`` GPUs of ``hbm_bytes`` each.  MoE models put their
    experts expert-parallel; ``attn`` picks their attention: ``"dp"`` (each GPU its own
    sequences, replicated attention weights) or ``"tp"`` (heads split over the GPUs)."""
    if n_gpus < 1:
        raise ValueError("need at least one GPU")
    w = weight_bytes(cfg, int8_projections=int8)
    usable = hbm_bytes - reserve_bytes - workspace_bytes
    p = Plan(n_gpus=n_gpus)
    L = cfg.num_hidden_layers
    if cfg.is_moe:
        ep = 1
        for d in range(1, n_gpus + 1):
            if n_gpus % d == 0 and cfg.num_experts % d == 0:
                ep = d
        p.ep, p.dp = ep, n_gpus // ep
        per_gpu = w.total - w.experts + w.experts // ep
        kv_heads = cfg.num_key_value_heads
        tp = _tp_degree_heads(cfg, ep) if attn == "tp" else 1
        if tp > 1:
            p.tp = tp
            sharded = w.attention + w.deltanet
            per_gpu -= sharded - sharded // tp
            kv_heads = max(1, cfg.num_key_value_heads // tp)
            p.notes.append(f"expert parallel {ep}: {cfg.num_experts // ep} experts per GPU, "
                           f"attention / DeltaNet heads tensor-parallel {tp}")
        else:
            p.notes.append(f"expert parallel {ep}: {cfg.num_experts // ep} experts per GPU, data-parallel attention")
    else:
        tp = _tp_degree(cfg, n_gpus)
        p.tp, p.dp = tp, n_gpus // tp
        sharded = w.attention + w.mlp + w.deltanet
        per_gpu = (w.total - sharded) + sharded // tp
        kv_heads = max(1, cfg.num_key_value_heads // tp)
        if tp > 1:
            p.notes.append(f"tensor parallel {tp} (sequence-parallel residual), {p.dp} replica(s)")
    if per_gpu > usable:
        # pipeline stages over replicas first: each stage holds a contiguous run of layers
        layer_bytes = (per_gpu - w.embed - w.lm_head) / max(1, L)
        while p.dp > 1 and per_gpu > usable:
            p.dp //= 2
            p.pp *= 2
            per_gpu = int(w.embed + w.lm_head + layer_bytes * -(-L // p.pp))
        if per_gpu > usable:
            fit_layers = max(0, int((usable - w.embed - w.lm_head) // max(1.0, layer_bytes)))
            p.offload_layers = max(0, -(-L // p.pp) - fit_layers)
            per_gpu = int(w.embed + w.lm_head + layer_bytes * (-(-L // p.pp) - p.offload_layers))
            p.notes.append(f"{p.offload_layers} layer(s) per stage streamed from pinned host memory")
        if p.pp > 1:
            p.notes.append(f"{p.pp} pipeline stages")
    base, extra = divmod(L, p.pp)
    p.layers_per_stage = [base + (1 if s < extra else 0) for s in range(p.pp)]
    p.weight_bytes_per_gpu = int(per_gpu)
    kv_room = max(0, usable - per_gpu)
    per_tok = kv_bytes_per_token(cfg, kv_heads) * max(p.layers_per_stage) // max(1, L)
    if per_tok:
        p.kv_blocks_per_gpu = kv_room // (per_tok * block_size)
        p.kv_tokens_per_gpu = p.kv_blocks_per_gpu * block_size
        p.kv_bytes_per_gpu = p.kv_blocks_per_gpu * per_tok * block_size
    p.fits = p.offload_layers == 0 and per_gpu <= usable
    return p
