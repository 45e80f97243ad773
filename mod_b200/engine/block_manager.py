"""Paged KV block allocator (block size 16) and recurrent-state slot pool.

A LIFO free list of physical block ids; a sequence owns the blocks listed in
its table.  Allocation failure returns False so the scheduler can preempt
instead of crashing (the reference has no KV allocator: its caches are
static per generate call, ``pio/models/qwen3_0_6b/architecture.py:195-201``).
"""
from __future__ import annotations

from typing import List

from .sequence import Sequence


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int = 16, max_seqs: int = 256):
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.free: List[int] = list(range(num_blocks - 1, -1, -1))
        self.free_slots: List[int] = list(range(max_seqs - 1, -1, -1))
        self.max_seqs = max_seqs

    @property
    def num_free(self) -> int:
        return len(self.free)

    def blocks_needed(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size

    def can_allocate(self, seq: Sequence, n_tokens: int) -> bool:
        need = self.blocks_needed(n_tokens) - len(seq.blocks)
        return need <= len(self.free) and (seq.state_slot >= 0 or self.free_slots)

    def allocate(self, seq: Sequence, n_tokens: int) -> bool:
        """Grow ``seq``'s table to hold ``n_tokens`` tokens."""
        if not self.can_allocate(seq, n_tokens):
            return False
        need = self.blocks_needed(n_tokens) - len(seq.blocks)
        for _ in range(max(0, need)):
            seq.blocks.append(self.free.pop())
        if seq.state_slot < 0:
            seq.state_slot = self.free_slots.pop()
        return True

    def release(self, seq: Sequence) -> None:
        self.free.extend(reversed(seq.blocks))
        seq.blocks = []
        if seq.state_slot >= 0:
            self.free_slots.append(seq.state_slot)
            seq.state_slot = -1
        seq.num_cached = 0

    def slot_of(self, seq: Sequence, pos: int) -> int:
        return seq.blocks[pos // self.block_size] * self.block_size + pos % self.block_size
