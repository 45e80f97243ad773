"""Model runner: turns a scheduled step into device tensors, runs the model,
samples, and brings the tokens back.

Per step the host builds the metadata (token ids, positions, KV slots, block
tables, context lengths) in pinned buffers, copies them to static device
buffers with one ``cudaMemcpyAsync`` each, runs the step, and copies the
sampled tokens back to pinned memory.  Decode steps replay a CUDA graph
captured once per padded batch size, so a step costs one graph launch plus
the two small copies.  The reference's "CUDA graph" wrapper is a no-op
(``pio/core/engine/backend.py:165-199``).
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch

from .batch import ForwardBatch
from .block_manager import BlockManager
from .sequence import Sequence


def _bucket(n: int, buckets: List[int]) -> int:
    for b in buckets:
        if n <= b:
            return b
    return n


class ModelRunner:
    def __init__(self, model, kv, states, blocks: BlockManager, max_batch: int, max_model_len: int,
                 use_graphs: bool = True, device=None):
        self.model, self.kv, self.states, self.blocks = model, kv, states, blocks
        self.device = torch.device(device) if device is not None else model.device
        self.max_batch = max_batch
        self.max_blocks = (max_model_len + blocks.block_size - 1) // blocks.block_size
        self.use_graphs = use_graphs and self.device.type == "cuda"
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_out: Dict[int, torch.Tensor] = {}
        self.buckets = sorted({b for b in (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 160, 192, 256) if b < max_batch}
                              | {max_batch})
        pin = self.device.type == "cuda"
        B, MB = max_batch, self.max_blocks
        # the dummy state slot for padded decode rows is the last one
        self.pad_slot = blocks.max_seqs
        self.h_ids = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        self.h_pos = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_slots = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_bt = torch.zeros(B, MB, dtype=torch.int32, pin_memory=pin)
        self.h_ctx = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_sslot = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        self.h_out = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        dev = self.device
        self.d_ids = torch.zeros(B, dtype=torch.long, device=dev)
        self.d_pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.d_slots = torch.zeros(B, dtype=torch.int32, device=dev)
        self.d_bt = torch.zeros(B, MB, dtype=torch.int32, device=dev)
        self.d_ctx = torch.zeros(B, dtype=torch.int32, device=dev)
        self.d_sslot = torch.zeros(B, dtype=torch.long, device=dev)
        self.d_lidx = torch.arange(B, dtype=torch.long, device=dev)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.sampler = None

    # ------------------------------------------------------------------ helpers
    def attn_splits(self, B: int) -> int:
        """Split-KV factor so that (sequences x KV heads x splits) fills the SMs."""
        if self.device.type != "cuda":
            return 1
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        ctas = max(1, B * self.model.Hkv)
        s = 1
        while ctas * s * 2 <= 2 * sms and s * 2 <= max(1, self.max_blocks // 8):
            s *= 2
        return s

    def _fb_decode(self, B: int) -> ForwardBatch:
        return ForwardBatch(input_ids=self.d_ids[:B], positions=self.d_pos[:B], slot_mapping=self.d_slots[:B],
                            block_tables=self.d_bt[:B], ctx_lens=self.d_ctx[:B], logits_idx=self.d_lidx[:B],
                            state_slots=self.d_sslot[:B], is_decode=True, attn_splits=self.attn_splits(B))

    def _copy_in(self, B: int) -> None:
        nb = 0
        for h, d in ((self.h_ids, self.d_ids), (self.h_pos, self.d_pos), (self.h_slots, self.d_slots),
                     (self.h_ctx, self.d_ctx), (self.h_sslot, self.d_sslot)):
            d[:B].copy_(h[:B], non_blocking=True)
            nb += h[:B].numel() * h.element_size()
        self.d_bt[:B].copy_(self.h_bt[:B], non_blocking=True)
        nb += self.h_bt[:B].numel() * 4
        self.h2d_bytes = nb

    def _sample(self, h: torch.Tensor, seqs: Optional[List[Sequence]] = None) -> torch.Tensor:
        if self.sampler is not None and seqs is not None and any(s.params.temperature > 0 for s in seqs):
            return self.sampler(self.model.logits(h), seqs)
        return self.model.sample_greedy(h)

    # ------------------------------------------------------------------ decode
    def _decode_body(self, B: int) -> torch.Tensor:
        h = self.model.forward(self._fb_decode(B), self.kv, self.states)
        return self.model.sample_greedy(h)

    def capture(self, B: int) -> None:
        """Captures the decode step for padded batch size ``B``."""
        torch.cuda.synchronize(self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        # pad rows: no KV write, empty context, dummy state slot
        self.d_slots[:B].fill_(-1)
        self.d_ctx[:B].zero_()
        self.d_sslot[:B].fill_(self.pad_slot)
        with torch.cuda.stream(s):
            for _ in range(2):
                self._decode_body(B)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = self._decode_body(B)
        torch.cuda.synchronize(self.device)
        self.graphs[B] = g
        self.graph_out[B] = out

    def decode(self, seqs: List[Sequence], return_logits: bool = False):
        n = len(seqs)
        B = _bucket(n, self.buckets) if self.use_graphs else n
        bs = self.blocks.block_size
        self.h_bt[:B].zero_()
        for i, s in enumerate(seqs):
            pos = s.length - 1
            self.h_ids[i] = s.all_tokens[-1]
            self.h_pos[i] = pos
            self.h_slots[i] = s.blocks[pos // bs] * bs + pos % bs
            self.h_ctx[i] = pos + 1
            self.h_sslot[i] = s.state_slot
            self.h_bt[i, :len(s.blocks)] = torch.tensor(s.blocks, dtype=torch.int32)
        for i in range(n, B):
            self.h_ids[i] = 0
            self.h_pos[i] = 0
            self.h_slots[i] = -1
            self.h_ctx[i] = 0
            self.h_sslot[i] = self.pad_slot
        self._copy_in(B)
        sampling = self.sampler is not None and any(s.params.temperature > 0 for s in seqs)
        if return_logits:
            h = self.model.forward(self._fb_decode(B), self.kv, self.states)
            for s in seqs:
                s.num_cached = s.length
            return self.model.logits(h)[:n].float()
        if self.use_graphs and not sampling:
            if B not in self.graphs:
                self._copy_in(B)
                self.capture(B)
                self._copy_in(B)
            self.graphs[B].replay()
            out = self.graph_out[B]
        else:
            h = self.model.forward(self._fb_decode(B), self.kv, self.states)
            out = self._sample(h, seqs + [seqs[0]] * (B - n))
        self.h_out[:B].copy_(out[:B], non_blocking=True)
        self.d2h_bytes = B * 8
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        for s in seqs:
            s.num_cached = s.length
        return self.h_out[:n].tolist()

    # ------------------------------------------------------------------ prefill
    def prefill(self, seqs: List[Sequence], query_lens: List[int], inputs_embeds=None, return_logits: bool = False):
        bs = self.blocks.block_size
        ids, pos, slots, ctx, lidx = [], [], [], [], []
        bt = torch.zeros(len(seqs), self.max_blocks, dtype=torch.int32)
        t = 0
        for i, (s, ql) in enumerate(zip(seqs, query_lens)):
            toks = s.all_tokens
            start = s.length - ql
            ids.extend(toks[start:])
            for p in range(start, s.length):
                pos.append(p)
                slots.append(s.blocks[p // bs] * bs + p % bs)
            ctx.append(s.length)
            t += ql
            lidx.append(t - 1)
            bt[i, :len(s.blocks)] = torch.tensor(s.blocks, dtype=torch.int32)
        dev = self.device
        pin = dev.type == "cuda"

        def up(x, dtype):
            h = torch.tensor(x, dtype=dtype)
            if pin:
                h = h.pin_memory()
            return h.to(dev, non_blocking=True)

        fb = ForwardBatch(input_ids=up(ids, torch.long), positions=up(pos, torch.int32),
                          slot_mapping=up(slots, torch.int32), block_tables=bt.to(dev),
                          ctx_lens=up(ctx, torch.int32), logits_idx=up(lidx, torch.long),
                          state_slots=up([s.state_slot for s in seqs], torch.long), is_decode=False,
                          query_lens=list(query_lens), ctx_lens_host=ctx, inputs_embeds=inputs_embeds)
        if self.states is not None:
            fresh = [s.state_slot for s, ql in zip(seqs, query_lens) if ql == s.length]
            if fresh:
                self.states.reset(torch.tensor(fresh, device=dev))
        h = self.model.forward(fb, self.kv, self.states)
        if return_logits:
            for s in seqs:
                s.num_cached = s.length
            return self.model.logits(h).float()
        out = self._sample(h, seqs).to("cpu")
        for s in seqs:
            s.num_cached = s.length
        return out.tolist()
