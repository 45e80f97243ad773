"""Per-kernel device-time table of a callable (torch profiler / CUPTI), used for
step breakdowns outside timed regions."""
from __future__ import annotations

import collections

import torch


def kernel_table(fn, reps: int = 3, top: int = 30) -> str:
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if e.device_type.name == "CUDA":
            n = e.name[:100]
            agg[n][0] += 1
            agg[n][1] += e.device_time_total
    tot = sum(v[1] for v in agg.values()) / reps
    lines = [f"total device us per call: {tot:.1f}"]
    for n, (c, t) in sorted(agg.items(), key=lambda x: -x[1][1])[:top]:
        lines.append(f"{t / reps:10.1f} us {c // reps:5d}x  {n}")
    return "\n".join(lines)
