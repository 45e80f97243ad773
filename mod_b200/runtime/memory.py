"""Unified memory manager: one owner of device memory per rank.

Regions: model weights, the paged KV block pool, communication buffers,
activations/workspace and a pinned host staging pool.  The manager sizes the
KV pool from what is left after weights (``plan_kv_blocks``), keeps a budget
per region, and swaps KV blocks of preempted sequences to pinned host memory
and back (:class:`KVSwapper`), so a preempted request can resume without
recomputing its prefix.

The reference's ``UnifiedMemoryManager`` keeps a byte budget and an LRU list
whose eviction is a no-op (``pio/common/memory/unified_manager.py:5-59``);
its ``MemoryManager`` only checks psutil pressure
(``pio/common/hardware/memory_manager.py:14-52``).
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch


@dataclass
class Region:
    name: str
    budget: int
    used: int = 0


class OutOfBudget(RuntimeError):
    pass


class UnifiedMemoryManager:
    def __init__(self, device="cuda", reserve_fraction: float = 0.05):
        self.device = torch.device(device)
        self.regions: Dict[str, Region] = OrderedDict()
        if self.device.type == "cuda":
            free, total = torch.cuda.mem_get_info(self.device)
        else:
            import psutil

            total = psutil.virtual_memory().total
            free = psutil.virtual_memory().available
        self.total = total
        self.free_at_start = free
        self.reserve = int(total * reserve_fraction)

    def define(self, name: str, budget: int) -> Region:
        r = Region(name, int(budget))
        self.regions[name] = r
        return r

    def charge(self, name: str, nbytes: int) -> None:
        r = self.regions[name]
        if r.used + nbytes > r.budget:
            raise OutOfBudget(f"region {name}: {r.used + nbytes} > budget {r.budget}")
        r.used += nbytes

    def release(self, name: str, nbytes: int) -> None:
        r = self.regions[name]
        r.used = max(0, r.used - nbytes)

    def plan_kv_blocks(self, bytes_per_block: int, weights_bytes: int, workspace_bytes: int = 2 << 30,
                       fraction: float = 0.9) -> int:
        """Blocks that fit after weights, workspace and the reserve."""
        avail = int((self.free_at_start - self.reserve - workspace_bytes) * fraction) - weights_bytes
        n = max(0, avail // max(1, bytes_per_block))
        self.define("kv", n * bytes_per_block)
        self.define("weights", weights_bytes)
        self.define("workspace", workspace_bytes)
        return n

    def report(self) -> Dict[str, Dict[str, int]]:
        return {r.name: {"budget": r.budget, "used": r.used} for r in self.regions.values()}


class PinnedPool:
    """Reusable pinned host buffers keyed by size (page-locked for async copies)."""

    def __init__(self, limit_bytes: int = 8 << 30):
        self.limit = limit_bytes
        self.used = 0
        self.free: Dict[int, List[torch.Tensor]] = {}

    def get(self, nbytes: int) -> torch.Tensor:
        lst = self.free.get(nbytes)
        if lst:
            return lst.pop()
        if self.used + nbytes > self.limit:
            raise OutOfBudget("pinned host pool exhausted")
        self.used += nbytes
        return torch.empty(nbytes, dtype=torch.uint8, pin_memory=torch.cuda.is_available())

    def put(self, buf: torch.Tensor) -> None:
        self.free.setdefault(buf.numel(), []).append(buf)


class KVSwapper:
    """Moves the KV blocks of a sequence between the device pool and pinned host memory."""

    def __init__(self, kv, pool: Optional[PinnedPool] = None):
        self.kv = kv
        self.pool = pool or PinnedPool()
        self.stream = torch.cuda.Stream() if torch.cuda.is_available() and kv.k and kv.k[0].is_cuda else None
        self.saved: Dict[int, List[torch.Tensor]] = {}
        self.external: set = set()   # requests whose saved blocks were handed in (``stage``), not pool buffers

    def _block_bytes(self) -> int:
        k = self.kv.k[0]
        return k[0].numel() * k.element_size()

    def swap_out(self, req_id: int, blocks: List[int]) -> None:
        bufs = []
        idx = torch.tensor(blocks, device=self.kv.k[0].device)
        if self.stream:  # after every kernel that wrote these blocks
            self.stream.wait_stream(torch.cuda.current_stream(self.kv.k[0].device))
        ctx = torch.cuda.stream(self.stream) if self.stream else _null()
        with ctx:
            for t in self.kv.k + self.kv.v:
                data = t.index_select(0, idx)
                host = self.pool.get(data.numel() * data.element_size()).view(data.dtype).view(data.shape)
                host.copy_(data, non_blocking=True)
                bufs.append(host)
        if self.stream:
            self.stream.synchronize()
        self.saved[req_id] = bufs

    def stage(self, req_id: int, bufs: List[torch.Tensor]) -> None:
        """Registers KV computed elsewhere (e.g. a context-parallel prefill) as the saved
        blocks of ``req_id``: one tensor per K layer then per V layer, each shaped like
        ``nblk`` blocks of that cache.  The next ``swap_in`` copies them into the
        sequence's blocks; they are not returned to the pinned pool."""
        if len(bufs) != len(self.kv.k) + len(self.kv.v):
            raise ValueError(f"stage: {len(bufs)} tensors for {len(self.kv.k)} K + {len(self.kv.v)} V layers")
        for t, b in zip(self.kv.k + self.kv.v, bufs):
            if tuple(b.shape[1:]) != tuple(t.shape[1:]):
                raise ValueError(f"stage: block shape {tuple(b.shape[1:])} != cache block {tuple(t.shape[1:])}")
        self.saved[req_id] = [b.to(self.kv.k[0].dtype) for b in bufs]
        self.external.add(req_id)

    def swap_in(self, req_id: int, blocks: List[int]) -> None:
        bufs = self.saved.pop(req_id)
        idx = torch.tensor(blocks[:bufs[0].shape[0]], device=self.kv.k[0].device)  # the saved blocks' new homes
        for t, host in zip(self.kv.k + self.kv.v, bufs):
            t.index_copy_(0, idx, host.to(t.device, non_blocking=True))
        if t.is_cuda:  # the host buffers go back to the pool only after the copies have read them
            torch.cuda.current_stream(t.device).synchronize()
        if req_id in self.external:
            self.external.discard(req_id)
            return
        for host in bufs:
            self.pool.put(host.view(torch.uint8).view(-1))

    def has(self, req_id: int) -> bool:
        return req_id in self.saved


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
