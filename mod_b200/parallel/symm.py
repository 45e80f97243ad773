"""Symmetric buffers bound to an NVLink multicast object (NVLS).

One allocation per rank, the same size and layout on every rank, mapped into
every peer (``peers``: each rank's unicast base in this process) and bound to
one multicast object (``mc``: its multicast base).  A ``multimem.st`` to
``mc + off`` lands at ``off`` in every rank's copy; a ``multimem.ld_reduce``
from ``mc + off`` returns the sum over the ranks' copies, computed in the
NVSwitch.  The allocation and the handle exchange are torch.distributed's
symmetric-memory plumbing (CUDA backend); the kernels that use the addresses
are this package's own (``csrc/cuda/tp_nvls.cu``).

Only ``multimem.*`` instructions may address the multicast range: no TMA or
bulk copy (with or without cluster multicast) and no library kernel is given
``mc`` or a peer's unicast address.
"""
from __future__ import annotations

import importlib

import torch
import torch.distributed as dist


def nvls_supported(group=None) -> bool:
    """True when every rank of ``group`` is a CUDA device with multicast support
    (symmetric memory importable and the driver reporting multicast)."""
    if not torch.cuda.is_available() or not dist.is_initialized() or dist.get_backend(group) != "nccl":
        return False
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
    except ImportError:
        return False
    from ..ops import load_extension

    try:
        ok = bool(load_extension().multicast_supported(torch.cuda.current_device()))
    except Exception:  # noqa: BLE001 - an extension without the query: no NVLS
        ok = False
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=torch.cuda.current_device())
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


class SymmetricBuffer:
    """``nbytes`` of zeroed symmetric memory per rank with a multicast mapping.

    ``peers`` is a device int64 tensor of every rank's unicast base address (the
    same form as :class:`mod_b200.parallel.ep.ExchangeBuffer`, so the P2P kernels
    run on it unchanged); ``mc`` is the multicast base (int)."""

    def __init__(self, nbytes: int, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        dev = torch.device("cuda", torch.cuda.current_device())
        try:
            symm_mem.set_backend("CUDA")
        except Exception:  # noqa: BLE001 - older releases have a single backend
            pass
        self.tensor = symm_mem.empty(int(nbytes), dtype=torch.uint8, device=dev)
        self.tensor.zero_()
        self.handle = symm_mem.rendezvous(self.tensor, self.group.group_name)
        base = int(self.handle.buffer_ptrs[self.rank])
        shift = self.tensor.data_ptr() - base  # the tensor may start inside the symmetric block
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if mc == 0:
            raise RuntimeError("SymmetricBuffer: no multicast mapping (NVLS unavailable on this system)")
        self.mc = mc + shift
        self.peers = torch.tensor([int(p) + shift for p in self.handle.buffer_ptrs], dtype=torch.int64, device=dev)
        self.own = self.tensor.data_ptr()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Every rank finishes its kernels before any rank lets the mapping go."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.handle = None
        self.tensor = None
