"""Qwen3-VL-style vision-language model.

Vision encoder (per image): pixels [3, S, S] -> 16x16 patches -> linear patch
embedding -> ViT blocks (pre-RMSNorm, bidirectional attention with 2-D RoPE:
half of each head's rotary pairs rotate with the patch row, half with the
column; GELU MLP) -> 2x2 spatial merge (4 neighbouring patches concatenated)
-> RMSNorm -> MLP projector -> LLM hidden size.  A 448x448 image gives
28x28 patches and 196 visual tokens.

The LLM is the dense decoder; a prompt holds ``image_token_id`` placeholders
(one per visual token) whose embeddings are replaced by the projected vision
features at prefill (``LLMEngine`` calls :meth:`VLModel.prefill_embeds`).

Reference: ``pio/models/qwen3_vl_2b/vision_transformer_kernels.py:26-149`` and
``pio/models/qwen3_vl_2b/model.py:45-253`` (patch 14, no 2-D RoPE, no merge,
no token interleave; visual features are added to early hidden states).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn.functional as F

from ..config.models import VisionConfig, VLConfig
from ..ops import reference as R
from .decoder import DecoderLM
from .weights import ModelWeights, _Init, random_weights


@dataclass
class ViTBlock:
    norm1: torch.Tensor
    qkv: torch.Tensor
    qkv_bias: torch.Tensor
    proj: torch.Tensor
    proj_bias: torch.Tensor
    norm2: torch.Tensor
    fc1: torch.Tensor
    fc1_bias: torch.Tensor
    fc2: torch.Tensor
    fc2_bias: torch.Tensor


@dataclass
class VisionWeights:
    patch: torch.Tensor          # [hidden, 3*p*p]
    patch_bias: torch.Tensor
    blocks: List[ViTBlock]
    merge_norm: torch.Tensor     # [4*hidden]
    merge_fc1: torch.Tensor      # [4*hidden, 4*hidden]
    merge_fc1_bias: torch.Tensor
    merge_fc2: torch.Tensor      # [out_hidden, 4*hidden]
    merge_fc2_bias: torch.Tensor


def random_vision_weights(vc: VisionConfig, device="cpu", dtype=torch.bfloat16, seed: int = 1) -> VisionWeights:
    ini = _Init(device, dtype, seed)
    H, F4 = vc.hidden_size, vc.intermediate_size
    blocks = [ViTBlock(norm1=ini.ones(H), qkv=ini.normal(3 * H, H), qkv_bias=ini.zeros(3 * H), proj=ini.normal(H, H),
                       proj_bias=ini.zeros(H), norm2=ini.ones(H), fc1=ini.normal(F4, H), fc1_bias=ini.zeros(F4),
                       fc2=ini.normal(H, F4), fc2_bias=ini.zeros(H)) for _ in range(vc.num_hidden_layers)]
    M = H * vc.spatial_merge_size ** 2
    return VisionWeights(patch=ini.normal(H, vc.in_channels * vc.patch_size ** 2), patch_bias=ini.zeros(H),
                         blocks=blocks, merge_norm=ini.ones(M), merge_fc1=ini.normal(M, M), merge_fc1_bias=ini.zeros(M),
                         merge_fc2=ini.normal(vc.out_hidden_size, M), merge_fc2_bias=ini.zeros(vc.out_hidden_size))


# ------------------------------------------------------------------ preprocessing
def preprocess(images: torch.Tensor, vc: VisionConfig, size: int) -> torch.Tensor:
    """[B, 3, h, w] float in [0, 1] -> resized to size x size, mean/std normalised,
    patchified in merge-group order -> [B, (size/p)^2, 3*p*p]."""
    x = images.float()
    if x.shape[-1] != size or x.shape[-2] != size:
        x = F.interpolate(x, size=(size, size), mode="bilinear", align_corners=False)
    mean = torch.tensor(vc.image_mean, device=x.device).view(1, 3, 1, 1)
    std = torch.tensor(vc.image_std, device=x.device).view(1, 3, 1, 1)
    x = (x - mean) / std
    return patchify(x, vc.patch_size, vc.spatial_merge_size)


def patchify(x: torch.Tensor, p: int, m: int) -> torch.Tensor:
    """[B, C, S, S] -> [B, N, C*p*p]; patches ordered so each 2x2 merge group is
    4 consecutive rows (grid row-major over groups, then within a group)."""
    B, C, S, _ = x.shape
    g = S // p
    t = x.view(B, C, g // m, m, p, g // m, m, p)            # b c GH mh ph GW mw pw
    t = t.permute(0, 2, 5, 3, 6, 1, 4, 7)                    # b GH GW mh mw c ph pw
    return t.reshape(B, g * g, C * p * p)


def grid_positions(S: int, p: int, m: int, device) -> torch.Tensor:
    """(row, col) of each patch in the merge-group order used by :func:`patchify`."""
    g = S // p
    r = torch.arange(g, device=device)
    rr, cc = torch.meshgrid(r, r, indexing="ij")
    pos = torch.stack([rr, cc], -1).view(g // m, m, g // m, m, 2).permute(0, 2, 1, 3, 4)
    return pos.reshape(g * g, 2)


def rope_2d(x: torch.Tensor, pos: torch.Tensor, theta: float = 10000.0) -> torch.Tensor:
    """x [N, heads, D]; first half of the rotary pairs follow the row index,
    second half the column index (rotate-half form)."""
    N, Hh, D = x.shape
    quarter = D // 4
    inv = 1.0 / (theta ** (torch.arange(quarter, device=x.device, dtype=torch.float32) / quarter))
    ang = torch.cat([pos[:, :1].float() * inv, pos[:, 1:].float() * inv], -1)   # [N, D/2]
    cos, sin = ang.cos()[:, None], ang.sin()[:, None]
    xf = x.float()
    x1, x2 = xf[..., : D // 2], xf[..., D // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)


# ------------------------------------------------------------------ encoder
def _linear_gelu(be, x, w, b):
    if hasattr(be, "linear_gelu"):
        return be.linear_gelu(x, w, b)
    h = be.linear(x, w, bias=b)
    return F.gelu(h.float(), approximate="tanh").to(x.dtype)


def vision_forward(vc: VisionConfig, vw: VisionWeights, patches: torch.Tensor, be, size: int,
                   stop_before_fc2: bool = False) -> torch.Tensor:
    """patches [B, N, 3*p*p] -> visual tokens [B, N/4, out_hidden] (backend ops, any dtype).
    ``stop_before_fc2`` returns the merger's hidden rows [B*N/4, M] before its last linear (the
    tensor-parallel path fuses that linear with the exchange of the rows)."""
    B, N, _ = patches.shape
    H, heads = vc.hidden_size, vc.num_attention_heads
    D = H // heads
    eps = vc.layer_norm_eps
    pos = grid_positions(size, vc.patch_size, vc.spatial_merge_size, patches.device)
    x = be.linear(patches.reshape(B * N, -1).to(vw.patch.dtype).contiguous(), vw.patch, bias=vw.patch_bias)
    native = getattr(be, "name", "") == "native" and D in (64, 128, 256) and patches.is_cuda
    if native:
        # every image is one sequence of a paged cache (block table = its own blocks), so one
        # bidirectional tcgen05 flash launch covers the whole batch
        nblk = (N + 15) // 16
        dev = patches.device
        bt = torch.arange(B * nblk, dtype=torch.int32, device=dev).view(B, nblk)
        cu = torch.arange(B + 1, dtype=torch.int32, device=dev) * N
        ctx = torch.full((B,), N, dtype=torch.int32, device=dev)
        pos_i = pos.int().contiguous()
        alloc = torch.empty if N % 16 == 0 else torch.zeros  # no stale NaNs behind the last patch
        kcache = alloc(B * nblk, heads, 16, D, dtype=torch.bfloat16, device=dev)
        vcache = alloc(B * nblk, heads, D, 16, dtype=torch.bfloat16, device=dev)
        q = torch.empty(B * N, heads * D, dtype=torch.bfloat16, device=dev)
    for blk in vw.blocks:
        h = be.rmsnorm(x, blk.norm1, eps)
        qkv = be.linear(h, blk.qkv, bias=blk.qkv_bias)
        if native:
            be.N.vit_rope_kv(qkv.contiguous(), pos_i, N, heads, D, 10000.0, q, kcache, vcache)
            o = be.N.attn_prefill_tc(q.view(B * N, heads, D), kcache, vcache, bt, cu, ctx, N, causal=False)
            o = o.reshape(B * N, H)
        else:
            qkv = qkv.view(B, N, 3, heads, D)
            outs = []
            for b in range(B):
                qb = rope_2d(qkv[b, :, 0], pos)
                kb = rope_2d(qkv[b, :, 1], pos)
                outs.append(R.attn_prefill(qb, kb, qkv[b, :, 2], causal=False))
            o = torch.stack(outs).reshape(B * N, H)
        x = be.linear(o, blk.proj, bias=blk.proj_bias, residual=x)
        h = be.rmsnorm(x, blk.norm2, eps)
        h = _linear_gelu(be, h, blk.fc1, blk.fc1_bias)
        x = be.linear(h, blk.fc2, bias=blk.fc2_bias, residual=x)
    m2 = vc.spatial_merge_size ** 2
    x = x.reshape(B * N // m2, m2 * H)                          # merge groups are consecutive rows
    x = be.rmsnorm(x.contiguous(), vw.merge_norm, eps)
    x = _linear_gelu(be, x, vw.merge_fc1, vw.merge_fc1_bias)
    if stop_before_fc2:
        return x.to(vw.merge_fc2.dtype).contiguous()
    x = be.linear(x.to(vw.merge_fc2.dtype), vw.merge_fc2, bias=vw.merge_fc2_bias)
    return x.view(B, N // m2, -1)


class VLModel:
    """Vision encoder + dense decoder, with the engine's prefill hook."""

    def __init__(self, cfg: VLConfig, text_weights: ModelWeights, vision_weights: VisionWeights, backend,
                 image_size: int = 448):
        self.cfg = cfg
        self.text = DecoderLM(cfg.text, text_weights, backend)
        self.vw = vision_weights
        self.be = backend
        self.image_size = image_size
        p, m = cfg.vision.patch_size, cfg.vision.spatial_merge_size
        self.tokens_per_image = (image_size // p) ** 2 // (m * m)
        # attributes the engine reads
        self.w, self.Hkv, self.device = self.text.w, self.text.Hkv, self.text.device

    def forward(self, fb, kv, states=None):
        return self.text.forward(fb, kv, states)

    def logits(self, h):
        return self.text.logits(h)

    def sample_greedy(self, h):
        return self.text.sample_greedy(h)

    def encode_images(self, images: torch.Tensor) -> torch.Tensor:
        vc = self.cfg.vision
        if getattr(self.be, "name", "") == "native" and images.is_cuda and len(vc.image_mean) <= 4:
            patches = self.be.N.patchify(images, self.image_size, vc.patch_size, vc.spatial_merge_size,
                                         vc.image_mean, vc.image_std)
        else:
            patches = preprocess(images, vc, self.image_size)
        return vision_forward(self.cfg.vision, self.vw, patches, self.be, self.image_size)

    def prompt_with_image(self, text_ids: List[int]) -> List[int]:
        return [self.cfg.image_token_id] * self.tokens_per_image + list(text_ids)

    def prefill_embeds(self, sched) -> Optional[torch.Tensor]:
        """Input embeddings for a prefill step; None when no sequence has an image."""
        seqs = [s for s in sched.seqs if s.images is not None]
        if not seqs:
            return None
        feats = self.encode_images(torch.stack([s.images for s in seqs]).to(self.device))
        by_seq = {s.req_id: feats[i] for i, s in enumerate(seqs)}
        rows = []
        for s, ql in zip(sched.seqs, sched.query_lens):
            toks = s.all_tokens[s.length - ql:]
            ids = torch.tensor(toks, device=self.device)
            e = self.be.embed(ids, self.w.embed)
            if s.req_id in by_seq:
                mask = ids == self.cfg.image_token_id
                n = int(mask.sum())
                if n:
                    f = by_seq[s.req_id]
                    # placeholders may be split across prefill chunks: skip the ones already consumed
                    start = sum(1 for t in s.all_tokens[: s.length - ql] if t == self.cfg.image_token_id)
                    e = e.clone()
                    e[mask] = f[start:start + n].to(e.dtype)
            rows.append(e)
        return torch.cat(rows, 0)


class TPVLModel:
    """Tensor-parallel vision-language model: the dense decoder is a
    :class:`TPDecoderLM` (sequence-parallel residual stream), the vision
    encoder runs data-parallel over the step's images (image j on rank
    j % world), and the merger's last linear is fused with the exchange: each
    visual row is stored straight into the shard of the rank that owns its token
    row (``FusedVisionExchange``: GEMM epilogue P2P stores + flags;
    ``NcclVisionExchange``: the all-gather baseline)."""

    def __init__(self, cfg: VLConfig, text_shard: ModelWeights, vision_weights: VisionWeights, backend, comm,
                 world: int, exchange, image_size: int = 448):
        from .tp_decoder import TPDecoderLM

        self.cfg = cfg
        self.text = TPDecoderLM(cfg.text, text_shard, backend, comm, world)
        self.vw, self.be, self.vx, self.world = vision_weights, backend, exchange, world
        self.rank = comm.rank
        self.image_size = image_size
        p, m = cfg.vision.patch_size, cfg.vision.spatial_merge_size
        self.tokens_per_image = (image_size // p) ** 2 // (m * m)
        self.w, self.Hkv, self.device = self.text.w, self.text.Hkv, self.text.device

    def forward(self, fb, kv, states=None):
        return self.text.forward(fb, kv, states)

    def logits(self, h):
        return self.text.logits(h)

    def sample_greedy(self, h):
        return self.text.sample_greedy(h)

    def prompt_with_image(self, text_ids: List[int]) -> List[int]:
        return [self.cfg.image_token_id] * self.tokens_per_image + list(text_ids)

    def _hidden(self, images: torch.Tensor) -> torch.Tensor:
        vc = self.cfg.vision
        if getattr(self.be, "name", "") == "native" and images.is_cuda:
            patches = self.be.N.patchify(images, self.image_size, vc.patch_size, vc.spatial_merge_size,
                                         vc.image_mean, vc.image_std)
        else:
            patches = preprocess(images, vc, self.image_size)
        return vision_forward(vc, self.vw, patches, self.be, self.image_size, stop_before_fc2=True)

    def prefill_embeds(self, sched) -> torch.Tensor:
        """This rank's shard [pr, H] of the step's input embeddings (text rows embedded here,
        image rows delivered by the exchange).  Every rank calls it for every prefill step."""
        from ..parallel.tp import padded_tokens

        img_tok, r, N = self.cfg.image_token_id, self.rank, self.world
        ids, vis = [], []          # vis: (global row, sequence index, feature index)
        img_order = []             # sequences with image rows in this step, in schedule order
        g = 0
        for i, (s, ql) in enumerate(zip(sched.seqs, sched.query_lens)):
            start = s.length - ql
            toks = s.all_tokens[start:]
            ids.extend(toks)
            if s.images is not None:
                before = sum(1 for t in s.all_tokens[:start] if t == img_tok)
                rows = [(g + k, before) for k, t in enumerate(toks) if t == img_tok]
                if rows:
                    img_order.append(i)
                    vis.extend((gr, i, before + j) for j, (gr, _) in enumerate(rows))
            g += ql
        T = g
        Tp = padded_tokens(T, N)
        pr = Tp // N
        dev = self.device
        idt = torch.tensor(ids + [0] * (Tp - T), dtype=torch.long, device=dev)
        h = self.be.embed(idt[r * pr:(r + 1) * pr].contiguous(), self.w.embed)
        mine = {i for j, i in enumerate(img_order) if j % N == r}
        sel = [(gr, i, f) for gr, i, f in vis if i in mine]
        my_rows = torch.tensor([gr - r * pr for gr, _, _ in vis if r * pr <= gr < (r + 1) * pr], dtype=torch.int32,
                               device=dev)
        if sel:
            order = sorted(mine)
            hid = self._hidden(torch.stack([sched.seqs[i].images for i in order]).to(dev))
            per = hid.shape[0] // len(order)
            pos = {i: k for k, i in enumerate(order)}
            idx = torch.tensor([pos[i] * per + f for _, i, f in sel], dtype=torch.long, device=dev)
            x = hid.index_select(0, idx).contiguous()
            row_map = torch.tensor([gr for gr, _, _ in sel], dtype=torch.int32, device=dev)
        else:
            x = torch.empty(0, self.vw.merge_fc2.shape[1], dtype=self.vw.merge_fc2.dtype, device=dev)
            row_map = torch.empty(0, dtype=torch.int32, device=dev)
        self.vx.exchange(x, self.vw.merge_fc2, self.vw.merge_fc2_bias, row_map, h, my_rows, pr)
        return h


def random_vl_weights(cfg: VLConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0):
    return random_weights(cfg.text, device=device, dtype=dtype, seed=seed), \
        random_vision_weights(cfg.vision, device=device, dtype=dtype, seed=seed + 1)


@torch.no_grad()
def oracle_forward(cfg: VLConfig, tw: ModelWeights, vw: VisionWeights, images: torch.Tensor, ids: torch.Tensor,
                   image_size: int) -> torch.Tensor:
    """fp32 reference: image tokens replaced by vision features, then the text oracle."""
    from . import oracle
    from .backend import TorchBackend

    f32 = lambda t: t.float() if isinstance(t, torch.Tensor) else t  # noqa: E731
    vw32 = VisionWeights(**{k: (f32(v) if not isinstance(v, list) else [ViTBlock(**{kk: f32(vv) for kk, vv in vars(b).items()}) for b in v])
                            for k, v in vars(vw).items()})
    feats = vision_forward(cfg.vision, vw32, preprocess(images, cfg.vision, image_size), TorchBackend(), image_size)
    emb = tw.embed.float()[ids]
    for b in range(ids.shape[0]):
        m = ids[b] == cfg.image_token_id
        emb[b, m] = feats[b, : int(m.sum())]
    return oracle.forward(cfg.text, tw, ids, inputs_embeds=emb)


# ------------------------------------------------------------------ plugin
from ..api.engine_plugin import EnginePlugin  # noqa: E402


class VisionLanguageEnginePlugin(EnginePlugin):
    """``infer((text_or_ids, pixels))`` for Qwen3-VL-style models."""

    image_size = 448

    def load_model(self, config=None):
        from ..engine.llm_engine import LLMEngine
        from .backend import make_backend

        rt = self.runtime
        dev = torch.device(rt["device"])
        dtype = torch.float32 if dev.type == "cpu" else torch.bfloat16
        cfg = self._full_config
        tw, vw = random_vl_weights(cfg, device=dev, dtype=dtype, seed=rt["seed"])
        be = make_backend(rt["backend"])
        self.vl = VLModel(cfg, tw, vw, be, image_size=rt.get("image_size", self.image_size))
        self.engine = LLMEngine(cfg.text, model=self.vl, backend=rt["backend"], device=dev,
                                max_batch=rt["max_batch"], max_model_len=max(rt["max_model_len"], 512),
                                use_graphs=rt.get("use_graphs"))
        return self.engine

    def infer(self, data):
        if isinstance(data, tuple) and len(data) == 2:
            text, pixels = data
            ids = self.tokenize(text) if isinstance(text, str) else [int(t) for t in text]
            prompt = self.vl.prompt_with_image(ids)
            rid = self.engine.add_request(prompt, self._params(ignore_eos=True), images=pixels)
            while self.engine.has_unfinished():
                self.engine.step()
            out = self.engine.seqs.pop(rid).output
            return self.detokenize(out) if isinstance(text, str) else prompt + out
        return super().infer(data)

    def encode_images(self, images):
        return self.vl.encode_images(images)
