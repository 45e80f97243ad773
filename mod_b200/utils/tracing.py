"""Tracing: NVTX ranges, on-demand torch.profiler traces, device-timed regions.

The reference times with wall clocks and psutil deltas
(``src/inference_pio/models/qwen3_0_6b/benchmarks/benchmark_inference.py:89-107``)
and has no trace export.  Here:

* ``nvtx_range(name)`` marks a region for Nsight timelines.  Disabled unless
  ``MB_NVTX=1`` or ``enable_nvtx(True)``; when disabled it costs one bool test,
  so the decoder keeps its per-layer ranges on the hot path.
* ``trace(path)`` records a torch.profiler trace (CPU + CUDA activity when a
  GPU is present) and writes it as a Chrome trace JSON.
* ``DeviceTimer`` times a region with CUDA events on the current stream and,
  under ``torch.distributed``, reports the maximum over ranks.
"""
from __future__ import annotations

import contextlib
import os
import time
from typing import Iterator, List, Optional

import torch

_NVTX = os.environ.get("MB_NVTX", "0") not in ("", "0", "false", "False")


def enable_nvtx(on: bool = True) -> None:
    global _NVTX
    _NVTX = bool(on)


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if not _NVTX:
        yield
        return
    pushed = False
    try:
        torch.cuda.nvtx.range_push(name)
        pushed = True
    except Exception:  # no CUDA runtime in this process: ranges are a no-op
        pass
    try:
        yield
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def trace(path: str, cuda: Optional[bool] = None, record_shapes: bool = False) -> Iterator[object]:
    """Profile the body with torch.profiler and export a Chrome trace to ``path``."""
    from torch.profiler import ProfilerActivity, profile

    if cuda is None:
        cuda = torch.cuda.is_available()
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if cuda else [])
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    with profile(activities=acts, record_shapes=record_shapes) as prof:
        yield prof
        if cuda:
            torch.cuda.synchronize()
    prof.export_chrome_trace(path)


class DeviceTimer:
    """Accumulates device time of repeated regions.

    On a GPU the region is bracketed by CUDA events on the current stream;
    without one, by ``perf_counter`` (CPU backends).  ``result_ms()``
    synchronises and, when a process group is initialised, returns the max
    over ranks (the slowest rank sets a collective step's time).
    """

    def __init__(self, device: Optional[torch.device] = None):
        self.cuda = torch.cuda.is_available() and (device is None or torch.device(device).type == "cuda")
        self._pairs: List[tuple] = []
        self._cpu_ms = 0.0
        self._t0 = 0.0

    @contextlib.contextmanager
    def region(self) -> Iterator[None]:
        if self.cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            yield
            b.record()
            self._pairs.append((a, b))
        else:
            t0 = time.perf_counter()
            yield
            self._cpu_ms += (time.perf_counter() - t0) * 1000.0
            self._pairs.append(None)

    @property
    def count(self) -> int:
        return len(self._pairs)

    def local_ms(self) -> float:
        if not self.cuda:
            return self._cpu_ms
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in self._pairs)

    def result_ms(self) -> float:
        ms = self.local_ms()
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            dev = torch.device("cuda", torch.cuda.current_device()) if self.cuda else torch.device("cpu")
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms
