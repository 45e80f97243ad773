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


class PrefixCachingBlockManager(BlockManager):
    """Block manager that shares the KV blocks of common prompt prefixes.

    A full block is identified by a hash chain over its tokens and every token
    before it, so equal hashes mean equal KV contents.  A new sequence adopts
    the longest chain of cached full blocks that matches its prompt (capped so
    the last prompt token is computed into a private block: shared blocks are
    never written), and its prefill starts after them.  Blocks are reference
    counted; a cached block whose last user finished stays in an LRU list and
    is reused by a later match or evicted when free blocks run out.  Sequences
    register their full blocks after each step (``register``).  Not for models
    with recurrent state or for image prompts: their state cannot be rebuilt
    from KV blocks alone, so the engine does not enable it there.
    """

    def __init__(self, num_blocks: int, block_size: int = 16, max_seqs: int = 256):
        super().__init__(num_blocks, block_size, max_seqs)
        from collections import OrderedDict

        self.cache: dict = {}            # chain hash -> block
        self.hash_of: dict = {}          # block -> chain hash (cached blocks only)
        self.ref: dict = {}              # cached block -> users
        self.lru: "OrderedDict[int, None]" = OrderedDict()   # cached blocks without users, oldest first
        self.hits = 0                    # blocks adopted from the cache
        self.queries = 0                 # full prompt blocks looked up

    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.lru)

    def _chain(self, tokens, n_blocks: int):
        bs, h, out = self.block_size, 0, []
        for i in range(n_blocks):
            h = hash((h, tuple(tokens[i * bs:(i + 1) * bs])))
            out.append(h)
        return out

    def _take(self) -> int:
        if self.free:
            return self.free.pop()
        b, _ = self.lru.popitem(last=False)        # evict the least recently released cached block
        del self.cache[self.hash_of.pop(b)]
        self.ref.pop(b, None)
        return b

    def _match(self, seq: Sequence) -> None:
        if seq.blocks or getattr(seq, "images", None) is not None:
            return
        n_full = (len(seq.prompt) - 1) // self.block_size
        self.queries += n_full
        for h in self._chain(seq.prompt, n_full):
            b = self.cache.get(h)
            if b is None:
                break
            if b in self.lru:
                del self.lru[b]
            self.ref[b] = self.ref.get(b, 0) + 1
            seq.blocks.append(b)
            self.hits += 1
        seq.num_cached = len(seq.blocks) * self.block_size
        seq.registered = len(seq.blocks)

    def can_allocate(self, seq: Sequence, n_tokens: int) -> bool:
        need = self.blocks_needed(n_tokens) - len(seq.blocks)
        return need <= self.num_free and (seq.state_slot >= 0 or bool(self.free_slots))

    def allocate(self, seq: Sequence, n_tokens: int) -> bool:
        fresh = not seq.blocks
        if fresh:
            self._match(seq)
        if not self.can_allocate(seq, n_tokens):
            if fresh and seq.blocks:           # undo the adoption: the sequence stays waiting
                self._drop(seq)
            return False
        for _ in range(max(0, self.blocks_needed(n_tokens) - len(seq.blocks))):
            seq.blocks.append(self._take())
        if seq.state_slot < 0:
            seq.state_slot = self.free_slots.pop()
        return True

    def _drop(self, seq: Sequence) -> None:
        for b in reversed(seq.blocks):
            if b in self.hash_of:
                self.ref[b] -= 1
                if self.ref[b] == 0:
                    self.lru[b] = None
            else:
                self.free.append(b)
        seq.blocks = []
        seq.num_cached = 0
        seq.registered = 0

    def release(self, seq: Sequence) -> None:
        self._drop(seq)
        if seq.state_slot >= 0:
            self.free_slots.append(seq.state_slot)
            seq.state_slot = -1

    def register(self, seq: Sequence) -> None:
        """Enter the sequence's full, computed blocks into the cache."""
        if getattr(seq, "images", None) is not None:
            return
        done = seq.num_cached // self.block_size
        start = getattr(seq, "registered", 0)
        if done <= start:
            return
        chain = self._chain(seq.all_tokens, done)
        for i in range(start, done):
            b, h = seq.blocks[i], chain[i]
            if b in self.hash_of or h in self.cache:
                continue                        # already shared, or the same content lives in another block
            self.cache[h] = b
            self.hash_of[b] = h
            self.ref[b] = 1
        seq.registered = done
