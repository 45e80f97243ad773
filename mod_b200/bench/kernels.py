"""Kernel microbenchmarks at the flagship (Qwen3-30B-A3B decode/prefill) shapes.

    python -m mod_b200.bench.kernels --case moe_gateup [--iters 20]

Each case builds its inputs once (weights rotated across copies when they
would fit in L2), captures ``iters`` launches in one CUDA graph after warm-up
and times its replay with CUDA events (so host dispatch cost, which dominates
a 5-15 us kernel launched from Python, is not in the number; ``--eager`` times
plain launches instead), and prints one JSON line: microseconds per launch, algorithmic bytes and
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


def case(name: str, T: int = 128):
    from ..ops import native as N

    dev = "cuda"
    bf = torch.bfloat16
    if name.startswith("cublas:"):  # the same GEMM shapes through torch.matmul (cuBLAS), for comparison
        K, Nn = {"qkv": (2048, 5120), "o": (4096, 2048), "lm_head": (2048, 151936),
                 "router": (2048, 128)}[name.split(":")[1]]
        ws = _rot(lambda: (torch.randn(Nn, K, device=dev) * 0.02).to(bf), K * Nn * 2)
        x = torch.randn(T, K, device=dev).to(bf)
        y = torch.empty(T, Nn, device=dev, dtype=bf)
        i = [0]

        def run():
            torch.matmul(x, ws[i[0] % len(ws)].t(), out=y)
            i[0] += 1
        return run, K * Nn * 2 + T * K * 2 + T * Nn * 2, 2 * T * K * Nn
    if name.startswith("clw8:"):  # int8-weight cluster GEMM: clw8:qkv, clw8:o
        from ..ops.quant import quantize_int8

        K, Nn = {"qkv": (2048, 5120), "o": (4096, 2048)}[name.split(":")[1]]
        ws = _rot(lambda: quantize_int8(torch.randn(Nn, K, device=dev) * 0.02), K * Nn)
        x = torch.randn(T, K, device=dev).to(bf)
        y = torch.empty(T, Nn, device=dev, dtype=bf)
        i = [0]

        def run():
            w = ws[i[0] % len(ws)]
            N.linear_cluster_w8(x, w.q, w.scale, out=y)
            i[0] += 1
        return run, K * Nn + Nn * 4 + T * K * 2 + T * Nn * 2, 2 * T * K * Nn
    if name.startswith("cl:"):  # cluster split-K GEMM (DSMEM reduction): cl:qkv, cl:o, cl:router[:cs]
        parts = name.split(":")
        K, Nn = {"qkv": (2048, 5120), "o": (4096, 2048), "router": (2048, 128)}[parts[1]]
        cs = int(parts[2]) if len(parts) > 2 else 0
        ws = _rot(lambda: (torch.randn(Nn, K, device=dev) * 0.02).to(bf), K * Nn * 2)
        x = torch.randn(T, K, device=dev).to(bf)
        y = torch.empty(T, Nn, device=dev, dtype=bf)
        i = [0]

        def run():
            N.linear_cluster(x, ws[i[0] % len(ws)], out=y, cs=cs)
            i[0] += 1
        return run, K * Nn * 2 + T * K * 2 + T * Nn * 2, 2 * T * K * Nn
    if name in ("qkv", "o", "lm_head", "router"):
        K, Nn = {"qkv": (2048, 5120), "o": (4096, 2048), "lm_head": (2048, 151936), "router": (2048, 128)}[name]
        ws = _rot(lambda: (torch.randn(Nn, K, device=dev) * 0.02).to(bf), K * Nn * 2)
        x = torch.randn(T, K, device=dev).to(bf)
        y = torch.empty(T, Nn, device=dev, dtype=bf)
        wsp = torch.empty(16 * T * Nn, device=dev)
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
        B, Hq, Hkv, D = (T if name == "attn_decode" else 128), 32, 4, 128
        ctx = 600 if name == "attn_decode" else 512
        nbps = (ctx + 15) // 16
        nb = B * nbps + 8
        kc = torch.randn(nb, Hkv, 16, D, device=dev).to(bf)
        vc = torch.randn(nb, Hkv, D, 16, device=dev).to(bf)
        bt = torch.randperm(nb - 8, device=dev)[: B * nbps].view(B, nbps).int().contiguous()
        cl = torch.full((B,), ctx, device=dev, dtype=torch.int32)
        kv_bytes = B * ctx * Hkv * D * 2 * 2
        if name == "attn_decode":  # the engine's own launch policy (chunking, split-KV combine)
            from ..models.backend import NativeBackend

            be = NativeBackend()
            q = torch.randn(B, Hq, D, device=dev).to(bf)
            return (lambda: be.attn_decode(q, kc, vc, bt, cl)), kv_bytes, 4 * B * Hq * ctx * D
        q = torch.randn(B * ctx, Hq, D, device=dev).to(bf)
        cu = torch.arange(B + 1, device=dev, dtype=torch.int32) * ctx
        flops = 4 * B * Hq * D * ctx * (ctx + 1) // 2
        return (lambda: N.attn_prefill_tc(q, kc, vc, bt, cu, cl, ctx)), kv_bytes + 2 * q.numel() * 2, flops
    if name.startswith(("lin:", "w8:")):  # ad-hoc shape: lin:T:K:N[:splits] (bf16) or w8:T:K:N (int8 weights)
        kind, T_, K, Nn, *sp = name.split(":")
        T_, K, Nn = int(T_), int(K), int(Nn)
        splits = int(sp[0]) if sp else -1
        x = torch.randn(T_, K, device=dev).to(bf)
        y = torch.empty(T_, Nn, device=dev, dtype=bf)
        wsp = torch.empty(8 * T_ * Nn, device=dev) if T_ <= 256 else None
        i = [0]
        if kind == "w8":
            from ..ops.quant import quantize_int8

            ws = _rot(lambda: quantize_int8(torch.randn(Nn, K, device=dev) * 0.02), K * Nn)

            def run():
                w = ws[i[0] % len(ws)]
                N.linear_w8(x, w.q, w.scale, out=y, workspace=wsp)
                i[0] += 1
            wbytes = K * Nn + 4 * Nn
        else:
            ws = _rot(lambda: (torch.randn(Nn, K, device=dev) * 0.02).to(bf), K * Nn * 2)

            def run():
                N.linear(x, ws[i[0] % len(ws)], out=y, workspace=wsp, splits=splits)
                i[0] += 1
            wbytes = K * Nn * 2
        return run, wbytes + T_ * K * 2 + T_ * Nn * 2, 2 * T_ * K * Nn
    if name in ("w8_qkv", "w8_prefill"):
        from ..ops.quant import quantize_int8

        T_, K, Nn = (128, 2048, 5120) if name == "w8_qkv" else (4096, 2048, 2048)
        ws = _rot(lambda: quantize_int8(torch.randn(Nn, K, device=dev) * 0.02), K * Nn)
        x = torch.randn(T_, K, device=dev).to(bf)
        y = torch.empty(T_, Nn, device=dev, dtype=bf)
        wsp = torch.empty(8 * T_ * Nn, device=dev) if T_ <= 256 else None
        i = [0]

        def run():
            w = ws[i[0] % len(ws)]
            N.linear_w8(x, w.q, w.scale, out=y, workspace=wsp)
            i[0] += 1
        return run, K * Nn + Nn * 4 + T_ * K * 2 + T_ * Nn * 2, 2 * T_ * K * Nn
    if name == "w8_moe_gateup":
        # Qwen3-Next experts: 512 experts, top-10, intermediate 512, hidden 2048; 128 tokens
        from ..ops.quant import quantize_int8

        E, I, H, k = 512, 512, 2048, 10
        rows = T * k
        counts = torch.full((E,), rows // E, dtype=torch.int32)
        counts[: rows - int(counts.sum())] += 1
        offs = torch.zeros(E + 1, dtype=torch.int32)
        offs[1:] = counts.cumsum(0)
        offs = offs.to(dev)
        w = quantize_int8(torch.randn(E * 2 * I, H, device=dev) * 0.02)
        xs = torch.randn(rows, H, device=dev).to(bf)
        out = torch.empty(rows, I, device=dev, dtype=bf)
        return ((lambda: N.linear_w8(xs, w.q, w.scale, out=out, offs=offs, groups=E, swiglu=True,
                                     max_rows_per_group=4)), E * 2 * I * H + E * 2 * I * 4, 2 * rows * H * 2 * I)
    if name in ("deltanet_decode", "deltanet_prefill"):
        # Qwen3-Next linear attention: 16 key heads, 32 value heads, d = 128, conv 4
        Hk, Hv, d = 16, 32, 128
        C = 2 * Hk * d + Hv * d
        S = 128
        conv = torch.zeros(S, C, 3, device=dev)
        ssm = torch.randn(S, Hv, d, d, device=dev) * 0.01
        cw = (torch.randn(C, 4, device=dev) * 0.3).to(bf)
        A = torch.zeros(Hv, device=dev)
        dtb = torch.zeros(Hv, device=dev)
        nw = torch.ones(d, device=dev, dtype=bf)
        if name == "deltanet_decode":
            B = 128
            mix = torch.randn(B, C, device=dev).to(bf)
            z = torch.randn(B, Hv * d, device=dev).to(bf)
            ba = torch.randn(B, 2 * Hv, device=dev).to(bf)
            slots = torch.arange(B, device=dev)
            out = torch.empty(B, Hv * d, device=dev, dtype=bf)
            nbytes = B * Hv * d * d * 4 * 2 + B * C * (2 + 4 * 2 + 3 * 8) + B * Hv * d * 4
            return ((lambda: N.deltanet_decode(mix, z, ba, cw, conv, ssm, slots, A, dtb, nw, Hk, Hv, d, d, 1e-6,
                                               out=out)), nbytes, B * Hv * d * d * 6)
        nseq, L = 4, int(os.environ.get("MB_BENCH_DN_LEN", "2048"))  # tokens per sequence
        Tt = nseq * L
        mix = torch.randn(Tt, C, device=dev).to(bf)
        z = torch.randn(Tt, Hv * d, device=dev).to(bf)
        ba = torch.randn(Tt, 2 * Hv, device=dev).to(bf)
        slots = torch.arange(nseq, device=dev)
        cu = torch.arange(nseq + 1, device=dev, dtype=torch.int32) * L
        seq_of = torch.arange(Tt, device=dev, dtype=torch.int32) // L
        out = torch.empty(Tt, Hv * d, device=dev, dtype=bf)
        xc = torch.empty(Tt, C, device=dev)
        return ((lambda: N.deltanet_prefill(mix, z, ba, cw, conv, ssm, slots, cu, seq_of, A, dtb, nw, Hk, Hv, d, d,
                                            1e-6, out=out, xc=xc)), Tt * C * (2 + 4 + 4) + Tt * Hv * d * 4,
                Tt * Hv * d * d * 6)
    if name == "rope_qknorm":  # Qwen3-30B-A3B decode: 32 q / 4 kv heads of 128, paged KV write
        from ..ops import reference as R

        Hq, Hkv, D = 32, 4, 128
        qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).to(bf)
        qw = torch.ones(D, device=dev, dtype=bf)
        kw = torch.ones(D, device=dev, dtype=bf)
        pos = torch.randint(0, 4096, (T,), device=dev, dtype=torch.int32)
        invf = R.inv_freq(D, 1e6, device=dev)
        nb = T + 8
        kc = torch.zeros(nb, Hkv, 16, D, device=dev, dtype=bf)
        vc = torch.zeros(nb, Hkv, D, 16, device=dev, dtype=bf)
        slots = (torch.randperm(nb - 1, device=dev)[:T] * 16).int()
        q = torch.empty(T, Hq, D, device=dev, dtype=bf)
        return ((lambda: N.rope_qknorm(qkv, qw, kw, pos, invf, slots, q, kc, vc, Hq, Hkv, D, D, 1e-6)),
                qkv.numel() * 2 * 2, 0)
    if name == "moe_route":  # softmax top-8 of 128 experts, counts / offsets / cursors
        E, k = 128, 8
        logits = torch.randn(T, E, device=dev).to(bf)
        ids = torch.empty(T, k, dtype=torch.int32, device=dev)
        wts = torch.empty(T, k, dtype=torch.float32, device=dev)
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        offs = torch.empty(E + 1, dtype=torch.int32, device=dev)
        cursor = torch.empty(E, dtype=torch.int32, device=dev)
        return ((lambda: N.moe_route(logits, k, True, ids, wts, counts, offs, cursor)),
                logits.numel() * 2 + T * k * 8, 0)
    if name in ("sample", "argmax"):  # T rows of the 151,936-entry vocabulary
        V = 151936
        logits = torch.randn(T, V, device=dev).to(bf)
        if name == "argmax":
            out = torch.empty(T, dtype=torch.long, device=dev)
            return (lambda: N.argmax(logits, out=out)), logits.numel() * 2, 0
        temp = torch.full((T,), 0.7, device=dev)
        tk = torch.full((T,), 50, device=dev, dtype=torch.int32)
        tp = torch.full((T,), 0.9, device=dev)
        seeds = torch.arange(T, device=dev, dtype=torch.int64)
        steps = torch.zeros(T, device=dev, dtype=torch.int64)
        out = torch.empty(T, dtype=torch.int64, device=dev)
        return (lambda: N.sample_tokens(logits, temp, tk, tp, seeds, steps, out=out)), logits.numel() * 2, 0
    if name == "embed":
        table = (torch.randn(151936, 2048, device=dev) * 0.02).to(bf)
        ids = torch.randint(0, 151936, (T,), device=dev)
        out = torch.empty(T, 2048, device=dev, dtype=bf)
        return (lambda: N.embed(ids, table, out=out)), T * 2048 * 2 * 2, 0
    if name == "patchify":  # 16 images 3 x 448 x 448 f32 -> 784 patches of 3*16*16 (merge-group order)
        imgs = torch.rand(16, 3, 448, 448, device=dev)
        out = torch.empty(16, 784, 768, device=dev, dtype=bf)
        mean, std = (0.48, 0.46, 0.41), (0.27, 0.26, 0.28)
        return (lambda: N.patchify(imgs, 448, 16, 2, mean, std, out=out)), imgs.numel() * 4 + out.numel() * 2, 0
    if name == "bias_gelu":  # ViT MLP up-projection output: 16 images x 784 patches x 4096
        y = torch.randn(16 * 784, 4096, device=dev).to(bf)
        b = torch.randn(4096, device=dev).to(bf)
        return (lambda: N.bias_act(y, b, True)), y.numel() * 2 * 2, 0
    if name == "rmsnorm":
        x = torch.randn(65536, 2048, device=dev).to(bf)
        w = torch.ones(2048, device=dev, dtype=bf)
        r = torch.randn_like(x)
        return (lambda: N.rmsnorm(x, w, 1e-6, residual=r)), x.numel() * 2 * 4, 0
    raise KeyError(name)


CASES = ["qkv", "o", "router", "lm_head", "moe_gateup", "moe_down", "attn_decode", "attn_prefill", "rmsnorm",
         "w8_qkv", "w8_prefill", "w8_moe_gateup", "deltanet_decode", "deltanet_prefill", "rope_qknorm", "moe_route",
         "sample", "argmax", "embed", "patchify", "bias_gelu"]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=128, help="decode tokens (T) of the GEMM / attention cases")
    ap.add_argument("--eager", action="store_true", help="time plain launches instead of a graph replay")
    a = ap.parse_args(argv)
    bw_peak, fl_peak, src = peaks()
    for name in (CASES if a.case == "all" else a.case.split(",")):
        run, nbytes, flops = case(name, a.tokens)
        for _ in range(a.warmup):
            run()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        if a.eager:
            s.record()
            for _ in range(a.iters):
                run()
            e.record()
        else:
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(g, stream=st):
                for _ in range(a.iters):
                    run()
            torch.cuda.synchronize()
            g.replay()  # warm
            torch.cuda.synchronize()
            s.record()
            g.replay()
            e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1000 / a.iters
        rec = {"case": name, "tokens": a.tokens, "us": round(us, 2), "bytes": nbytes, "flops": flops,
               "TBps": round(nbytes / us / 1e6, 3), "TFLOPs": round(flops / us / 1e6, 2),
               "frac_bw": round(nbytes / us / 1e6 / (bw_peak / 1e12), 3),
               "frac_tc": round(flops / us / 1e6 / (fl_peak / 1e12), 3), "peaks": src,
               "timing": "eager launches" if a.eager else "CUDA-graph replay"}
        print(json.dumps(rec), flush=True)
        del run
        torch.cuda.empty_cache()
    from ..ops import check_status

    check_status()


if __name__ == "__main__":
    main()
