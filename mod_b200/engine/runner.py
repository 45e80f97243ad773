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

import os

from typing import Dict, List, Optional

import numpy as np
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
        # numpy views of the pinned buffers: whole-slice writes from Python lists (one call per
        # field instead of one tensor indexing op per sequence)
        self.n_ids, self.n_pos, self.n_slots = self.h_ids.numpy(), self.h_pos.numpy(), self.h_slots.numpy()
        self.n_bt, self.n_ctx, self.n_sslot = self.h_bt.numpy(), self.h_ctx.numpy(), self.h_sslot.numpy()
        # (req_id, generation, blocks written) of each block-table row; a sequence's generation
        # changes whenever it is prefilled from scratch (new blocks after a preemption)
        self._bt_rows: List[tuple] = [(-1, 0, 0)] * B
        self._gen: Dict[int, int] = {}

    # ------------------------------------------------------------------ helpers
    def attn_splits(self, B: int) -> int:
        """Split-KV factor so that (sequences x KV heads x splits) fills the SMs."""
        if self.device.type != "cuda":
            return 1
        forced = int(os.environ.get("MB_ATTN_SPLITS", "0") or 0)  # fixed factor, for A/B timing
        if forced > 0:
            return max(1, min(forced, self.max_blocks))
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

    def _prepare_decode(self, seqs: List[Sequence], B: Optional[int] = None) -> int:
        """Fills the pinned step buffers for ``seqs`` and copies them to the
        device; returns the padded batch size (``B``, or the graph bucket)."""
        n = len(seqs)
        if B is None:
            B = _bucket(n, self.buckets) if self.use_graphs else n
        bs = self.blocks.block_size
        pos = [s.length - 1 for s in seqs]
        self.n_ids[:n] = [s.last_token for s in seqs]
        self.n_pos[:n] = pos
        self.n_slots[:n] = [s.blocks[p // bs] * bs + p % bs for s, p in zip(seqs, pos)]
        self.n_ctx[:n] = [p + 1 for p in pos]
        self.n_sslot[:n] = [s.state_slot for s in seqs]
        rows, gen = self._bt_rows, self._gen
        for i, s in enumerate(seqs):  # a row changes only when its sequence or block count does
            nb = len(s.blocks)
            key = (s.req_id, gen.get(s.req_id, 0))
            old = rows[i]
            if old[:2] != key:
                self.n_bt[i, :] = 0
                self.n_bt[i, :nb] = s.blocks
            elif old[2] != nb:  # blocks only grow while decoding
                self.n_bt[i, old[2]:nb] = s.blocks[old[2]:]
                if nb < old[2]:
                    self.n_bt[i, nb:old[2]] = 0
            rows[i] = key + (nb,)
        if B > n:  # padded rows: no KV write, empty context, dummy state slot
            self.n_ids[n:B] = 0
            self.n_pos[n:B] = 0
            self.n_slots[n:B] = -1
            self.n_ctx[n:B] = 0
            self.n_sslot[n:B] = self.pad_slot
            for i in range(n, B):
                if rows[i] != (-1, 0, 0):
                    self.n_bt[i, :] = 0
                    rows[i] = (-1, 0, 0)
        self._copy_in(B)
        return B

    def bucket_index(self, n: int) -> int:
        """Index in ``buckets`` of the padded decode batch size for ``n`` sequences."""
        b = _bucket(n, self.buckets)
        return self.buckets.index(b) if b in self.buckets else len(self.buckets) - 1

    def needs_sampling(self, seqs: List[Sequence]) -> bool:
        return self.sampler is not None and any(s.params.temperature > 0 for s in seqs)

    def idle_step(self, eager: bool = False) -> None:
        """A decode forward of padding rows only (no KV write, empty context, the dummy state
        slot) whose only effect is taking part in the expert-parallel exchanges of a step that
        the other ranks run: the smallest captured graph, or (``eager``) one row outside it."""
        graphs = self.use_graphs and not eager
        B = self.buckets[0] if graphs else 1
        self.n_ids[:B] = 0
        self.n_pos[:B] = 0
        self.n_slots[:B] = -1
        self.n_ctx[:B] = 0
        self.n_sslot[:B] = self.pad_slot
        for i in range(B):
            if self._bt_rows[i] != (-1, 0, 0):
                self.n_bt[i, :] = 0
                self._bt_rows[i] = (-1, 0, 0)
        self._copy_in(B)
        if graphs:
            self.graphs[B].replay()
        else:
            self.model.forward(self._fb_decode(B), self.kv, self.states)
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()

    def decode(self, seqs: List[Sequence], return_logits: bool = False, eager: bool = False):
        """``eager``: run the forward outside the captured graphs (expert-parallel steps in
        which another rank prefills)."""
        n = len(seqs)
        graphs = self.use_graphs and not eager
        B = _bucket(n, self.buckets) if graphs else n
        B = self._prepare_decode(seqs, B)
        sampling = self.needs_sampling(seqs)
        if return_logits:
            h = self.model.forward(self._fb_decode(B), self.kv, self.states)
            for s in seqs:
                s.num_cached = s.length
            return self.model.logits(h)[:n].float()
        if graphs and not sampling:
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

    def device_stepper(self, seqs: List[Sequence]):
        """Greedy decode steps that run entirely on the device, for timing.

        Returns a callable; each call replays the captured decode step for
        ``seqs`` and then advances every live row by one token on the device
        (next input = sampled token, position and context + 1, KV slot from the
        block table), so consecutive calls decode at a growing context with no
        host work in between.  The caller must have grown every sequence's
        block table to cover the positions the calls will reach.  The host-side
        sequences are not updated: the next ``decode`` rewrites every row."""
        assert self.use_graphs, "device steps replay the captured decode graph"
        n = len(seqs)
        B = self._prepare_decode(seqs)
        if B not in self.graphs:
            self.capture(B)
            self._copy_in(B)
        g, out, bs = self.graphs[B], self.graph_out[B], self.blocks.block_size
        native = getattr(self.model.be, "name", "") == "native"
        if native:
            from ..ops import load_extension

            C = load_extension()

            def step():
                g.replay()
                C.decode_advance(out, self.d_ids, self.d_pos, self.d_ctx, self.d_slots, self.d_bt, n, bs)
        else:  # library-only arm: the same update as torch ops
            rows = torch.arange(n, device=self.device)

            def step():
                g.replay()
                self.d_ids[:n].copy_(out[:n])
                self.d_pos[:n] += 1
                self.d_ctx[:n] += 1
                p = self.d_pos[:n].long()
                self.d_slots[:n] = (self.d_bt[rows, p // bs] * bs + p % bs).int()
        return step

    # ------------------------------------------------------------------ prefill
    def prefill(self, seqs: List[Sequence], query_lens: List[int], inputs_embeds=None, return_logits: bool = False):
        bs = self.blocks.block_size
        ids, pos, slots, ctx, lidx = [], [], [], [], []
        bt = np.zeros((len(seqs), self.max_blocks), dtype=np.int32)
        t = 0
        ends = []
        for i, (s, ql) in enumerate(zip(seqs, query_lens)):
            # the chunk covers positions [num_cached, num_cached + ql): the whole rest of the prompt,
            # or one chunk of it under chunked prefill
            start = s.num_cached
            end = start + ql
            assert 0 < end <= s.length, (start, ql, s.length)
            if start == 0:  # from scratch: fresh blocks, so cached block-table rows are stale
                self._gen[s.req_id] = self._gen.get(s.req_id, 0) + 1
            ids.append(np.asarray(s.all_tokens[start:end], dtype=np.int64))
            p = np.arange(start, end, dtype=np.int64)   # positions of the new tokens
            blk = np.asarray(s.blocks, dtype=np.int64)
            pos.append(p)
            slots.append(blk[p // bs] * bs + p % bs)
            ctx.append(end)
            ends.append(end)
            t += ql
            lidx.append(t - 1)
            bt[i, :len(s.blocks)] = s.blocks
        ids, pos, slots = np.concatenate(ids), np.concatenate(pos), np.concatenate(slots)
        dev = self.device
        pin = dev.type == "cuda"

        def up(x, dtype):
            h = torch.from_numpy(x).to(dtype) if isinstance(x, np.ndarray) else torch.tensor(x, dtype=dtype)
            if pin:
                h = h.pin_memory()
            return h.to(dev, non_blocking=True)

        fb = ForwardBatch(input_ids=up(ids, torch.long), positions=up(pos, torch.int32),
                          slot_mapping=up(slots, torch.int32), block_tables=up(bt, torch.int32),
                          ctx_lens=up(ctx, torch.int32), logits_idx=up(lidx, torch.long),
                          state_slots=up([s.state_slot for s in seqs], torch.long), is_decode=False,
                          query_lens=list(query_lens), ctx_lens_host=ctx, inputs_embeds=inputs_embeds)
        if self.states is not None:
            fresh = [s.state_slot for s in seqs if s.num_cached == 0]
            if fresh:
                self.states.reset(torch.tensor(fresh, device=dev))
        h = self.model.forward(fb, self.kv, self.states)
        if return_logits:
            for s, e in zip(seqs, ends):
                s.num_cached = e
            return self.model.logits(h).float()
        out = self._sample(h, seqs).to("cpu")
        for s, e in zip(seqs, ends):
            s.num_cached = e
        return out.tolist()
