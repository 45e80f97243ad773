"""Process-group plumbing: one process per GPU, ``torch.distributed`` for
rendezvous, handle exchange and the baseline collectives.

The reference has no distributed layer at all (its TP/EP settings are
config strings only: ``pio/models/glm_4_7_flash/config.py:108-111``).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    backend: str = "none"

    @property
    def is_dist(self) -> bool:
        return self.world > 1


def init(backend: Optional[str] = None, timeout_s: float = 120.0) -> DistInfo:
    """Initialises the default process group from torchrun's environment.
    Uses NCCL when CUDA is available (device bound to LOCAL_RANK), else gloo."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return DistInfo(0, 1, local, "none")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if not dist.is_initialized():
        import datetime

        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return DistInfo(rank, world, local, backend)


def info() -> DistInfo:
    if not dist.is_available() or not dist.is_initialized():
        return DistInfo()
    return DistInfo(dist.get_rank(), dist.get_world_size(), int(os.environ.get("LOCAL_RANK", "0")),
                    dist.get_backend())


def max_over_ranks(x: float, device=None) -> float:
    """Max of a host scalar over all ranks (device-timed numbers are reported this way)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    dev = device if device is not None else ("cuda" if dist.get_backend() == "nccl" else "cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
