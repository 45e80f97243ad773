"""Continuous-batching scheduler.

Each step is either a prefill step (new prompts, up to a token budget) or a
decode step (one token for every running sequence).  Prefill is preferred
while KV blocks and batch slots allow admission; when a decode step cannot
get a block for every sequence, the most recently admitted sequence is
preempted: with a swap hook (the engine's ``KVSwapper``) its KV blocks are
copied to pinned host memory, its device blocks freed, and it re-enters the
running set later by copying them back into fresh blocks, with no
recomputation; without one, its blocks are freed and it is re-queued for
recomputation.

The reference's ``BatchManager.step`` runs one request's full ``generate`` at
a time, with no batching (``pio/common/managers/batch_manager.py:40-84``), and
its ``AdaptiveBatchManager`` only tunes a batch-size number
(``pio/common/processing/adaptive_batch_manager.py:42-251``).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from typing import Optional, Deque, List

from .block_manager import BlockManager
from .sequence import Sequence, SeqStatus


@dataclass
class ScheduledStep:
    seqs: List[Sequence]
    is_decode: bool
    query_lens: List[int]


class Scheduler:
    def __init__(self, blocks: BlockManager, max_batch: int = 256, max_prefill_tokens: int = 16384,
                 prefill_chunk: Optional[int] = None):
        self.blocks = blocks
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.waiting: Deque[Sequence] = deque()
        self.running: List[Sequence] = []
        self.num_preempted = 0
        # chunked prefill: a prompt is computed prefill_chunk tokens per step, and prefill chunks
        # alternate with decode steps of the sequences already generating
        self.prefill_chunk = prefill_chunk
        self._last_prefill = False
        # KV swap hooks (set by the engine): on_preempt(seq) -> True when the sequence's KV was saved;
        # on_resume(seq) copies it back into the sequence's (new) blocks
        self.on_preempt = None
        self.on_resume = None
        self.num_swapped_out = 0
        self.num_resumed = 0

    def add(self, seq: Sequence) -> None:
        seq.status = SeqStatus.WAITING
        self.waiting.append(seq)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def _admit(self) -> List[Sequence]:
        picked: List[Sequence] = []
        budget = self.max_prefill_tokens
        while self.waiting and len(self.running) + len(picked) < self.max_batch:
            seq = self.waiting[0]
            if seq.swapped:  # resumes by swap-in (``_resume_swapped``), never by a prefill
                break
            n = seq.length if not self.prefill_chunk else min(seq.length, self.prefill_chunk)  # this step's tokens
            if picked and n > budget:
                break
            # reserve room for the whole prompt plus the first decode token
            if not self.blocks.allocate(seq, seq.length + 1):
                if not picked and not self.running and self.blocks.num_free == self.blocks.num_blocks:
                    # can never fit: fail it instead of spinning
                    self.waiting.popleft()
                    seq.status = SeqStatus.FAILED
                    seq.error = "prompt does not fit in the KV cache"
                    continue
                break
            self.waiting.popleft()
            picked.append(seq)
            budget -= n
        return picked

    @staticmethod
    def _partial(s: Sequence) -> bool:
        # one uncached prompt token left is decode-ready: decoding it equals prefilling it
        return s.num_cached < s.length - 1

    def _schedule_chunked(self) -> Optional[ScheduledStep]:
        part = [s for s in self.running if self._partial(s)]
        ready = [s for s in self.running if not self._partial(s)]
        if part and not (self._last_prefill and ready):
            budget, picked, qls = self.max_prefill_tokens, [], []
            for s in part:
                q = min(s.length - s.num_cached, self.prefill_chunk, budget)
                if q <= 0:
                    break
                picked.append(s)
                qls.append(q)
                budget -= q
            self._last_prefill = True
            return ScheduledStep(picked, False, qls)
        if not (self._last_prefill and ready):
            new = self._admit()
            if new:
                for s in new:
                    s.status = SeqStatus.RUNNING
                self.running.extend(new)
                self._last_prefill = True
                return ScheduledStep(new, False, [min(s.length - s.num_cached, self.prefill_chunk) for s in new])
        self._last_prefill = False
        return None

    def _resume_swapped(self) -> None:
        """Swapped-out sequences at the head of the queue rejoin the running set when their
        blocks (plus one decode slot) fit; their KV is copied back, no prefill needed."""
        while self.waiting and self.waiting[0].swapped and len(self.running) < self.max_batch:
            seq = self.waiting[0]
            cached = seq.num_cached
            if not self.blocks.allocate(seq, seq.length + 1):
                break
            self.waiting.popleft()
            self.on_resume(seq)
            seq.num_cached = cached
            seq.swapped = False
            seq.status = SeqStatus.RUNNING
            self.running.append(seq)
            self.num_resumed += 1

    def schedule(self) -> ScheduledStep:
        self._resume_swapped()
        if self.prefill_chunk:
            st = self._schedule_chunked()
            if st is not None:
                return st
            return self._decode_step()
        new = self._admit()
        if new:
            for s in new:
                s.status = SeqStatus.RUNNING
            self.running.extend(new)
            return ScheduledStep(new, False, [s.length - s.num_cached for s in new])
        return self._decode_step()

    def _decode_step(self) -> ScheduledStep:
        # decode: every running sequence needs a slot for one more token
        i = 0
        while i < len(self.running):
            seq = self.running[i]
            if self.blocks.allocate(seq, seq.length + 1):
                i += 1
                continue
            victim = self.running.pop()          # newest admitted
            cached = victim.num_cached
            swapped = (self.on_preempt is not None and not self._partial(victim) and self.on_preempt(victim))
            self.blocks.release(victim)
            if swapped:
                victim.num_cached = cached
                victim.swapped = True
                self.num_swapped_out += 1
            victim.status = SeqStatus.WAITING
            self.waiting.appendleft(victim)
            self.num_preempted += 1
        ready = [s for s in self.running if not self._partial(s)]
        return ScheduledStep(ready, True, [1] * len(ready))

    def finish(self, seq: Sequence, status: SeqStatus = SeqStatus.FINISHED) -> None:
        seq.status = status
        if seq in self.running:
            self.running.remove(seq)
        self.blocks.release(seq)
