"""Hardware backend plugins and device probing.

* :class:`CudaSm100Backend` - a B200 (sm_100) device: device info (SM count,
  HBM, clocks, peer-access matrix), allocation/copies through torch, matmul
  through the tcgen05 GEMM.
* :class:`CpuBackend` - the C++/OpenMP CPU library.

Replaces the reference's CUDA/CPU/OpenCL backend plugins
(``pio/plugins/cuda/base.py:9-96``, ``pio/plugins/cpu/base.py:8-59``) and its
hardware analyzer (``pio/common/hardware/hardware_analyzer.py:14-49``).
OpenCL/AMD/Intel backends are out of scope on B200; third-party backends
register through :func:`register_backend`.
"""
from __future__ import annotations

import os
import platform
from typing import Any, Callable, Dict, List

import torch

from .interfaces import HardwareBackendInterface


def _driver_attribute(index: int, name: str):
    """A CUDA driver device attribute read through cuda-python (None when unavailable)."""
    try:
        try:
            from cuda.bindings import driver as drv
        except ImportError:  # older cuda-python layout
            from cuda import cuda as drv
        err, = drv.cuInit(0)
        if int(err) != 0:
            return None
        err, dev = drv.cuDeviceGet(index)
        if int(err) != 0:
            return None
        err, val = drv.cuDeviceGetAttribute(getattr(drv.CUdevice_attribute, name), dev)
        return int(val) if int(err) == 0 else None
    except Exception:
        return None


def probe_system() -> Dict[str, Any]:
    """Host + device topology (no NVML needed)."""
    info: Dict[str, Any] = {"platform": platform.platform(), "cpu_count": os.cpu_count(),
                            "cuda_available": torch.cuda.is_available(), "devices": []}
    try:
        import psutil

        info["host_memory_gb"] = round(psutil.virtual_memory().total / 2**30, 1)
    except Exception:  # pragma: no cover
        pass
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            info["devices"].append({"index": i, "name": p.name, "sm": f"{p.major}.{p.minor}",
                                    "multiprocessors": p.multi_processor_count,
                                    "memory_gb": round(p.total_memory / 2**30, 1),
                                    # NVLink multicast objects (NVLS): the in-switch reduction path
                                    "multicast_supported": _driver_attribute(
                                        i, "CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED")})
        info["peer_access"] = [[i == j or torch.cuda.can_device_access_peer(i, j) for j in range(n)]
                               for i in range(n)]
    return info


class CudaSm100Backend(HardwareBackendInterface):
    name = "cuda"

    def __init__(self, index: int = 0):
        self.index = index
        self.device = torch.device("cuda", index)

    def initialize(self) -> bool:
        if not torch.cuda.is_available():
            return False
        p = torch.cuda.get_device_properties(self.index)
        self.supported = (p.major, p.minor) >= (10, 0)
        if self.supported:
            from ..ops import load_extension

            load_extension()
        return self.supported

    def get_device_info(self) -> Dict[str, Any]:
        p = torch.cuda.get_device_properties(self.index)
        free, total = torch.cuda.mem_get_info(self.index)
        return {"name": p.name, "compute_capability": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
                "memory_total_gb": round(total / 2**30, 1), "memory_free_gb": round(free / 2**30, 1)}

    def allocate(self, nbytes: int):
        return torch.empty(nbytes, dtype=torch.uint8, device=self.device)

    def memcpy_h2d(self, dst, src) -> None:
        dst.copy_(src, non_blocking=True)

    def memcpy_d2h(self, dst, src) -> None:
        dst.copy_(src)

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.device)

    def matmul(self, a, b):
        """a [M, K] @ b [K, N] in bf16 through the tcgen05 GEMM."""
        from ..ops import native

        return native.linear(a.to(torch.bfloat16).contiguous(), b.t().to(torch.bfloat16).contiguous())


class CpuBackend(HardwareBackendInterface):
    name = "cpu"

    def initialize(self) -> bool:
        import importlib

        try:
            self.C = importlib.import_module("mod_b200._cpu")
        except ImportError:
            return False
        return True

    def get_device_info(self) -> Dict[str, Any]:
        return {"name": platform.processor() or "cpu", "threads": self.C.get_max_threads()}

    def allocate(self, nbytes: int):
        return torch.empty(nbytes, dtype=torch.uint8)

    def memcpy_h2d(self, dst, src) -> None:
        dst.copy_(src)

    def memcpy_d2h(self, dst, src) -> None:
        dst.copy_(src)

    def matmul(self, a, b):
        a = a.float().contiguous()
        y = torch.empty(a.shape[0], b.shape[1])
        self.C.linear(a, b.t().float().contiguous(), y)
        return y


_REGISTRY: Dict[str, Callable[..., HardwareBackendInterface]] = {"cuda": CudaSm100Backend, "cpu": CpuBackend}


def register_backend(name: str, factory: Callable[..., HardwareBackendInterface]) -> None:
    _REGISTRY[name] = factory


def available_backends() -> List[str]:
    out = []
    for name in _REGISTRY:
        if name == "cuda":
            out += [f"cuda:{i}" for i in range(torch.cuda.device_count())] if torch.cuda.is_available() else []
        else:
            out.append(name)
    return out


def create_backend(spec: str) -> HardwareBackendInterface:
    kind, _, idx = spec.partition(":")
    if kind not in _REGISTRY:
        raise KeyError(f"unknown backend {spec!r}")
    return _REGISTRY[kind](int(idx)) if idx else _REGISTRY[kind]()
