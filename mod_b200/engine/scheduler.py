"""Continuous-batching scheduler.

Each step is either a prefill step (new prompts, up to a token budget) or a
decode step (one token for every running sequence).  Prefill is preferred
while KV blocks and batch slots allow admission; when a decode step cannot
get a block for every sequence, the most recently admitted sequence is
preempted (blocks freed, sequence re-queued for recomputation).

The reference's ``BatchManager.step`` runs one request's full ``generate`` at
a time, with no batching (``pio/common/managers/batch_manager.py:40-84``), and
its ``AdaptiveBatchManager`` only tunes a batch-size number
(``pio/common/processing/adaptive_batch_manager.py:42-251``).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from typing import Deque, List

from .block_manager import BlockManager
from .sequence import Sequence, SeqStatus


@dataclass
class ScheduledStep:
    seqs: List[Sequence]
    is_decode: bool
    query_lens: List[int]


class Scheduler:
    def __init__(self, blocks: BlockManager, max_batch: int = 256, max_prefill_tokens: int = 16384):
        self.blocks = blocks
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.waiting: Deque[Sequence] = deque()
        self.running: List[Sequence] = []
        self.num_preempted = 0

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
            n = seq.length
            if picked and n > budget:
                break
            # reserve room for the prompt plus the first decode token
            if not self.blocks.allocate(seq, n + 1):
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

    def schedule(self) -> ScheduledStep:
        new = self._admit()
        if new:
            for s in new:
                s.status = SeqStatus.RUNNING
            self.running.extend(new)
            return ScheduledStep(new, False, [s.length - s.num_cached for s in new])
        # decode: every running sequence needs a slot for one more token
        i = 0
        while i < len(self.running):
            seq = self.running[i]
            if self.blocks.allocate(seq, seq.length + 1):
                i += 1
                continue
            victim = self.running.pop()          # newest admitted
            self.blocks.release(victim)
            victim.status = SeqStatus.WAITING
            self.waiting.appendleft(victim)
            self.num_preempted += 1
        return ScheduledStep(list(self.running), True, [1] * len(self.running))

    def finish(self, seq: Sequence, status: SeqStatus = SeqStatus.FINISHED) -> None:
        seq.status = status
        if seq in self.running:
            self.running.remove(seq)
        self.blocks.release(seq)
