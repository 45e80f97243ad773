"""Per-step metrics and device timing.

``StepTimer`` brackets work with CUDA events on the launching stream and
reports device milliseconds (max over ranks when distributed);
``ServingMetrics`` aggregates TTFT / TPOT / throughput / occupancy records and
writes benchmark JSON that keeps the reference's result field names
(``benchmark_results/real_model_benchmarks_*.json``: avg_inference_time,
std, avg_memory_usage, peak_memory_usage, tokens_per_second, num_runs,
successful_runs) next to this engine's own.
"""
from __future__ import annotations

import json
import statistics
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch


class StepTimer:
    def __init__(self, device=None):
        self.cuda = torch.cuda.is_available() and (device is None or torch.device(device).type == "cuda")
        self.ms: List[float] = []

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize()
            self.s = torch.cuda.Event(enable_timing=True)
            self.e = torch.cuda.Event(enable_timing=True)
            self.s.record()
        else:
            self.t0 = time.perf_counter()
        return self

    def __exit__(self, *a):
        if self.cuda:
            self.e.record()
            torch.cuda.synchronize()
            ms = self.s.elapsed_time(self.e)
        else:
            ms = (time.perf_counter() - self.t0) * 1000
        from ..parallel.dist import max_over_ranks

        self.ms.append(max_over_ranks(ms))


@dataclass
class ServingMetrics:
    ttft_s: List[float] = field(default_factory=list)
    tpot_s: List[float] = field(default_factory=list)
    step_s: List[float] = field(default_factory=list)
    tokens: int = 0
    runs: int = 0
    failed: int = 0
    peak_memory_gb: float = 0.0

    def record_sequence(self, seq) -> None:
        self.runs += 1
        if seq.error:
            self.failed += 1
            return
        if seq.ttft is not None:
            self.ttft_s.append(seq.ttft)
        if seq.t_finish and seq.t_first_token and len(seq.output) > 1:
            self.tpot_s.append((seq.t_finish - seq.t_first_token) / (len(seq.output) - 1))
        self.tokens += len(seq.output)

    def summary(self, wall_s: Optional[float] = None) -> Dict[str, float]:
        def p(xs, q):
            return sorted(xs)[int(q * (len(xs) - 1))] if xs else float("nan")

        if torch.cuda.is_available():
            self.peak_memory_gb = torch.cuda.max_memory_allocated() / 2**30
        lat = self.ttft_s
        return {"avg_inference_time": statistics.mean(lat) if lat else float("nan"),
                "std": statistics.pstdev(lat) if len(lat) > 1 else 0.0,
                "avg_memory_usage": self.peak_memory_gb, "peak_memory_usage": self.peak_memory_gb,
                "tokens_per_second": (self.tokens / wall_s) if wall_s else float("nan"),
                "num_runs": self.runs, "successful_runs": self.runs - self.failed,
                "ttft_p50_s": p(self.ttft_s, 0.5), "ttft_p99_s": p(self.ttft_s, 0.99),
                "tpot_p50_s": p(self.tpot_s, 0.5)}

    def write_json(self, path: str, wall_s: Optional[float] = None, **extra) -> None:
        with open(path, "w") as f:
            json.dump({**self.summary(wall_s), **extra}, f, indent=2)
