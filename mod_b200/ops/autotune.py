"""GEMM launch-configuration cache: measured (split-K, orientation) per shape.

The reference's auto-tuner times one naive matmul with CUDA events and keeps a
JSON of tile sizes that its kernels never read
(``src/inference_pio/common/optimization/auto_tuner.py:7-40``,
``src/inference_pio/plugins/cuda/base.py:34-43``).  Here the cache drives the
tcgen05 GEMM: for a shape ``(T, N, K)`` (T activation rows, N output
features, K reduction) ``tune_linear`` times every legal pair of

* orientation -- 0: activations on the 128-row MMA side; 1: weights on it
  (swap-AB, legal for T <= 256 and N % 128 == 0), and
* split-K factor -- 1, 2, 4, 8, 16 (fp32 partials + a reduction kernel),

with CUDA events over a rotating set of weight copies larger than L2 (so every
launch streams its weights from HBM, as in a real decode step), and records the
fastest.  ``activate(cache)`` makes ``ops.native.linear`` use the cached pair
whenever its caller leaves both choices automatic; shapes not in the cache keep
the built-in heuristic.  The JSON is keyed by device name so one file can hold
entries for several GPU kinds.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterable, List, Optional, Tuple

import torch

Shape = Tuple[int, int, int]
_ACTIVE: Optional[Dict[Shape, Tuple[int, int]]] = None
SPLITS = (1, 2, 4, 8, 16)
_L2_BYTES = 126 * 1024 * 1024


class TuneCache:
    def __init__(self, path: Optional[str] = None, device_name: Optional[str] = None):
        self.path = path
        self.device_name = device_name or (torch.cuda.get_device_name() if torch.cuda.is_available() else "cpu")
        self.data: Dict[str, Dict[str, dict]] = {}
        if path and os.path.exists(path):
            with open(path) as f:
                self.data = json.load(f)

    @staticmethod
    def key(shape: Shape) -> str:
        return "%d,%d,%d" % shape

    def entries(self) -> Dict[str, dict]:
        return self.data.setdefault(self.device_name, {})

    def get(self, shape: Shape) -> Optional[dict]:
        return self.data.get(self.device_name, {}).get(self.key(shape))

    def put(self, shape: Shape, splits: int, orient: int, us: float, trials: Dict[str, float]) -> None:
        self.entries()[self.key(shape)] = {"splits": int(splits), "orient": int(orient), "us": round(us, 3),
                                           "trials": {k: round(v, 3) for k, v in trials.items()}}

    def table(self) -> Dict[Shape, Tuple[int, int]]:
        out = {}
        for k, v in self.data.get(self.device_name, {}).items():
            t, n, kk = (int(s) for s in k.split(","))
            out[(t, n, kk)] = (int(v["splits"]), int(v["orient"]))
        return out

    def save(self, path: Optional[str] = None) -> None:
        path = path or self.path
        if not path:
            raise ValueError("no path to save the tuning cache to")
        d = os.path.dirname(os.path.abspath(path))
        os.makedirs(d, exist_ok=True)
        tmp = path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(self.data, f, indent=1, sort_keys=True)
        os.replace(tmp, path)


def activate(cache: Optional[TuneCache]) -> None:
    """Route automatic GEMM launches through ``cache`` (None turns the cache off)."""
    global _ACTIVE
    _ACTIVE = None if cache is None else cache.table()


def lookup(T: int, N: int, K: int) -> Optional[Tuple[int, int]]:
    if _ACTIVE is None:
        return None
    return _ACTIVE.get((T, N, K))


def candidates(T: int, N: int, K: int) -> List[Tuple[int, int]]:
    """Legal (splits, orient) pairs for the tcgen05 linear kernel."""
    out = [(1, 0)]
    if T <= 256 and N % 128 == 0:
        kb = (K + 63) // 64
        out += [(s, 1) for s in SPLITS if s <= max(1, kb // 2)]
    return out


def _time_us(fn, reps: int) -> float:
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for i in range(reps):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000.0 / reps


def tune_linear(T: int, N: int, K: int, cache: TuneCache, reps: int = 20, warmup: int = 3,
                device: str = "cuda") -> dict:
    """Time every legal (splits, orient) for ``y[T,N] = x[T,K] @ w[N,K]^T`` and store the best."""
    from . import native

    global _ACTIVE
    prev = _ACTIVE
    activate(None)  # time the kernel's own choices, not a cached one
    try:
        g = torch.Generator(device=device).manual_seed(0)
        x = (torch.randn(T, K, device=device, generator=g) * 0.5).bfloat16()
        wbytes = N * K * 2
        copies = max(1, min(64, -(-2 * _L2_BYTES // wbytes)))
        ws_list = [(torch.randn(N, K, device=device, generator=g) * 0.02).bfloat16() for _ in range(copies)]
        y = torch.empty(T, N, dtype=torch.bfloat16, device=device)
        wsp = torch.empty(max(SPLITS) * T * N, dtype=torch.float32, device=device)
        trials: Dict[str, float] = {}
        for splits, orient in candidates(T, N, K):
            def run(i, s=splits, o=orient):
                native.linear(x, ws_list[i % copies], out=y, workspace=wsp, splits=s, orient=o)
            for i in range(warmup):
                run(i)
            trials[f"s{splits}o{orient}"] = _time_us(run, reps)
        best = min(trials, key=trials.get)
        s, o = int(best[1:best.index("o")]), int(best[best.index("o") + 1:])
        cache.put((T, N, K), s, o, trials[best], trials)
        return cache.get((T, N, K))
    finally:
        _ACTIVE = prev


def model_linear_shapes(cfg, tokens: Iterable[int]) -> List[Shape]:
    """The dense (non-grouped) projection shapes of one decoder at the given token counts."""
    H = cfg.hidden_size
    shapes = set()
    for T in tokens:
        if cfg.num_attention_heads:
            q_rows = cfg.num_attention_heads * cfg.head_dim * (2 if getattr(cfg, "attn_output_gate", False) else 1)
            shapes.add((T, q_rows + 2 * cfg.num_key_value_heads * cfg.head_dim, H))
            shapes.add((T, H, cfg.num_attention_heads * cfg.head_dim))
        if not getattr(cfg, "num_experts", 0):
            shapes.add((T, H, cfg.intermediate_size))
    return sorted(s for s in shapes if s[2] % 8 == 0)


def _activate_from_env() -> None:
    path = os.environ.get("MB_TUNE_CACHE", "")
    if path and os.path.exists(path):
        activate(TuneCache(path))


_activate_from_env()
