"""Kernel entry points.

``mod_b200.ops.native`` wraps the sm_100a extension (``mod_b200._C``);
``mod_b200.ops.reference`` holds plain PyTorch restatements of every op,
which serve as the fp32 oracle in tests and as the PyTorch+cuBLAS+NCCL
baseline path.  There is no silent fallback: on a machine with a CUDA device
``native`` raises if the extension cannot be imported.
"""
from __future__ import annotations

import importlib

import torch

_C = None
_err = None


def load_extension():
    """Imports ``mod_b200._C``; raises with the import error if it is missing."""
    global _C, _err
    if _C is not None:
        return _C
    try:
        _C = importlib.import_module("mod_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _err = e
        raise RuntimeError(
            "mod_b200 CUDA extension is not built (run `python setup.py build_ext --inplace`): %r" % (e,)
        ) from e
    return _C


def extension_available() -> bool:
    try:
        load_extension()
        return True
    except RuntimeError:
        return False


def check_status(device=None) -> None:
    """Raises if a kernel on ``device`` recorded an error (timeout, overflow...)."""
    C = load_extension()
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    code = C.read_and_clear_status(dev)
    if code:
        names = {1: "mbarrier wait timed out", 2: "peer flag wait timed out", 3: "index out of bounds",
                 4: "routing capacity exceeded"}
        raise RuntimeError(f"mod_b200 kernel status {code}: {names.get(code, 'unknown error')}")
