"""Kernel microbenchmarks at the flagship (Qwen3-30B-A3B decode/prefill) shapes.

    python -m mod_b200.bench.kernels --case moe_gateup [--iters 20]

Each case builds its inputs once (weights rotated across copies when they
would fit in L2), times ``iters`` launches with CUDA events after warm-up,
and prints one JSON line: microseconds per launch, algorithmic bytes and
FLOPs, achieved bandwidth / throughput and the fraction of the measured
peaks (``MEASURED_PEAKS.json`` when present, else 6.65 TB/s and
1.59 PFLOP/s).  The same cases are what the committed ncu summaries profile.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

HERE = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    return 6.65e12, 1.59e15, "fallback"


def _rot(make, nbytes, limit=512e6):
    n = max(1, int(limit // max(1, nbytes)))
    return [make() for _ in range(n)]


def case(name: str):
    from ..ops import native as N

    dev = "cuda"
    bf = torch.bfloat16
    T = 128
    if name in ("qkv", "o", "lm_head", "router"):
        K, Nn = {"qkv": (2048, 5120), "o": (4096, 2048), "lm_head": (2048, 151936), "router": (2048, 128)}[name]
        ws = _rot(lambda: (torch.randn(Nn, K, device=dev) * 0.02).to(bf), K * Nn * 2)
        x = torch.randn(T, K, device=dev).to(bf)
        y = torch.empty(T, Nn, device=dev, dtype=bf)
        wsp = torch.empty(8 * T * Nn, device=dev)
        orient = 0 if name == "lm_head" else -1
        i = [0]

        def run():
            N.linear(x, ws[i[0] % len(ws)], out=y, workspace=wsp, orient=orient)
            i[0] += 1
        return run, K * Nn * 2 + T * K * 2 + T * Nn * 2, 2 * T * K * Nn
    if name in ("moe_gateup", "moe_down"):
        E, I, H, k = 128, 768, 2048, 8
        counts = torch.full((E,), T * k // E, dtype=torch.int32)
        offs = torch.zeros(E + 1, dtype=torch.int32)
        offs[1:] = counts.cumsum(0)
        offs = offs.to(dev)
        if name == "moe_gateup":
            w = (torch.randn(E * 2 * I, H, device=dev) * 0.02).to(bf)
            xs = torch.randn(T * k, H, device=dev).to(bf)
            out = torch.empty(T * k, I, device=dev, dtype=bf)
            return (lambda: N.grouped_linear(xs, w, offs, E, True, 32, out=out)), w.numel() * 2, 2 * T * k * H * 2 * I
        w = (torch.randn(E * H, I, device=dev) * 0.02).to(bf)
        xs = torch.randn(T * k, I, device=dev).to(bf)
        out = torch.empty(T * k, H, device=dev, dtype=bf)
        return (lambda: N.grouped_linear(xs, w, offs, E, False, 32, out=out)), w.numel() * 2, 2 * T * k * H * I
    if name in ("attn_decode", "attn_prefill"):
        B, Hq, Hkv, D = 128, 32, 4, 128
        ctx = 600 if name == "attn_decode" else 512
        nbps = (ctx + 15) // 16
        nb = B * nbps + 8
        kc = torch.randn(nb, Hkv, 16, D, device=dev).to(bf)
        vc = torch.randn(nb, Hkv, D, 16, device=dev).to(bf)
        bt = torch.randperm(nb - 8, device=dev)[: B * nbps].view(B, nbps).int().contiguous()
        cl = torch.full((B,), ctx, device=dev, dtype=torch.int32)
        kv_bytes = B * ctx * Hkv * D * 2 * 2
        if name == "attn_decode":
            q = torch.randn(B, Hq, D, device=dev).to(bf)
            ws = torch.empty(B * Hq * 4 * (D + 1), device=dev)
            return (lambda: N.attn_decode_tc(q, kc, vc, bt, cl, splits=1, workspace=ws)), kv_bytes, 4 * B * Hq * ctx * D
        q = torch.randn(B * ctx, Hq, D, device=dev).to(bf)
        cu = torch.arange(B + 1, device=dev, dtype=torch.int32) * ctx
        flops = 4 * B * Hq * D * ctx * (ctx + 1) // 2
        return (lambda: N.attn_prefill_tc(q, kc, vc, bt, cu, cl, ctx)), kv_bytes + 2 * q.numel() * 2, flops
    if name == "rmsnorm":
        x = torch.randn(65536, 2048, device=dev).to(bf)
        w = torch.ones(2048, device=dev, dtype=bf)
        r = torch.randn_like(x)
        return (lambda: N.rmsnorm(x, w, 1e-6, residual=r)), x.numel() * 2 * 4, 0
    raise KeyError(name)


CASES = ["qkv", "o", "router", "lm_head", "moe_gateup", "moe_down", "attn_decode", "attn_prefill", "rmsnorm"]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    bw_peak, fl_peak, src = peaks()
    for name in (CASES if a.case == "all" else a.case.split(",")):
        run, nbytes, flops = case(name)
        for _ in range(a.warmup):
            run()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for _ in range(a.iters):
            run()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1000 / a.iters
        rec = {"case": name, "us": round(us, 2), "bytes": nbytes, "flops": flops,
               "TBps": round(nbytes / us / 1e6, 3), "TFLOPs": round(flops / us / 1e6, 2),
               "frac_bw": round(nbytes / us / 1e6 / (bw_peak / 1e12), 3),
               "frac_tc": round(flops / us / 1e6 / (fl_peak / 1e12), 3), "peaks": src}
        print(json.dumps(rec), flush=True)
        del run
        torch.cuda.empty_cache()
    from ..ops import check_status

    check_status()


if __name__ == "__main__":
    main()
