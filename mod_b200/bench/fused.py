"""Fused compute + collective paths against their rooflines (multi-GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m mod_b200.bench.fused [--case ep,tp] [--iters 50]

Each case times ``iters`` back-to-back replays of one call captured in a CUDA
graph (the NCCL baselines: eager calls) with CUDA events after warm-up, takes
the max over ranks, and prints one JSON line with the achieved time, the
roofline time max(T_c, T_m, T_n) and their ratio:

* T_c = FLOPs / measured bf16 GEMM peak
* T_m = HBM bytes (weights read once) / measured copy bandwidth
* T_n = bytes that must leave this GPU over NVLink / 770 GB/s (measured peer copy)

Cases:

* ``ep``   one Qwen3-30B-A3B MoE layer at decode (global batch 128, T = 128/N
  tokens per rank): router GEMM + top-8 + P2P dispatch + grouped expert GEMMs +
  P2P combine (``FusedEPMoE``), and the exchange kernels alone; the NCCL
  all-to-all baseline (``NcclEPMoE``) on the same shapes.
* ``tp``   one Qwen3-8B decoder layer's four boundaries at decode (T = 64):
  AG->QKV GEMM, o GEMM->RS(+residual+RMSNorm+push), AG->gate/up GEMM(+SwiGLU),
  down GEMM->RS (``FusedTP``); the NCCL + cuBLAS baseline (``NcclTP``).

Peaks come from ``MEASURED_PEAKS.json`` when present (else 6.65 TB/s and
1.59 PFLOP/s).  Synthetic N(0, 0.02) weights, random activations.
"""
from __future__ import annotations

import argparse
import os
import json

import torch
import torch.distributed as dist

from .kernels import peaks

NVLINK_BPS = 770e9
PROFILE = {"on": False, "tables": []}


def _dist() -> bool:
    return dist.is_initialized() and dist.get_world_size() > 1


def _barrier():
    if _dist():
        dist.barrier()


def _time(fn, iters, warmup=5, graph=True):
    """Device time per call, max over ranks.  graph=True captures one call in a CUDA graph and
    times replays (how the decode step runs), so host launch cost is not measured."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    _barrier()
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        fn = g.replay
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        _barrier()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1000 / iters
    if PROFILE["on"] and graph:  # every rank replays (kernels wait on peers); rank 0's table is printed
        from .profile import kernel_table

        _barrier()
        PROFILE["tables"].append(kernel_table(fn, 5, top=16))
    if not _dist():
        return us
    t = torch.tensor([us], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def _line(case, impl, us, flops, hbm, nvl, world, extra=None):
    bw, fl, src = peaks()
    tc, tm, tn = flops / fl * 1e6, hbm / bw * 1e6, nvl / NVLINK_BPS * 1e6
    roof = max(tc, tm, tn)
    d = {"case": case, "impl": impl, "n_gpus": world, "us": round(us, 2), "roofline_us": round(roof, 2),
         "frac_of_roofline": round(roof / us, 3), "T_c_us": round(tc, 2), "T_m_us": round(tm, 2),
         "T_n_us": round(tn, 2), "flops": flops, "hbm_bytes": hbm, "nvlink_bytes": nvl, "peaks": src}
    if extra:
        d.update(extra)
    return d


def case_ep(iters, rank, world, dev):
    from ..config import get_preset
    from ..models.backend import NativeBackend, TorchBackend
    from ..models.weights import MoEWeights
    from ..parallel.ep import FusedEPMoE, NcclEPMoE

    cfg = get_preset("qwen3-30b-a3b")
    H, I, E, K = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts, cfg.num_experts_per_tok
    El = E // world
    T = 128 // world
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    bf = torch.bfloat16
    mo = MoEWeights(router=(torch.randn(E, H, device=dev, generator=g) * 0.02).to(bf),
                    w13=(torch.randn(El * 2 * I, H, device=dev, generator=g) * 0.02).to(bf),
                    w2=(torch.randn(El * H, I, device=dev, generator=g) * 0.02).to(bf),
                    e_lo=rank * El, e_hi=(rank + 1) * El)
    x = torch.randn(T, H, device=dev, generator=g).to(bf)
    flops = 2 * T * K * H * 3 * I + 2 * T * H * E
    hbm = El * 3 * H * I * 2 + E * H * 2
    # tokens whose expert lives elsewhere leave this GPU, and their results come back
    nvl = 2 * T * K * H * 2 * (world - 1) // world
    out = []
    fused = FusedEPMoE(cfg, NativeBackend(), max_tokens=T)
    us = _time(lambda: fused(x, mo), iters)
    out.append(_line("ep_moe_layer", "fused", us, flops, hbm, nvl, world, {"tokens_per_rank": T, "experts_per_rank": El}))
    # the exchange alone: dispatch + combine without the expert GEMMs in between
    ctx = fused.small
    C, N = fused.C, fused.N
    logits = fused.be.linear(x, mo.router)
    ids = torch.empty(T, K, dtype=torch.int32, device=dev)
    wts = torch.empty(T, K, dtype=torch.float32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offs_g = torch.empty(E + 1, dtype=torch.int32, device=dev)
    cursor = torch.empty(E, dtype=torch.int32, device=dev)
    N.moe_route(logits, K, cfg.norm_topk_prob, ids, wts, counts, offs_g, cursor)
    emap = torch.empty(T * K, dtype=torch.int32, device=dev)
    y = torch.empty(world * ctx.cap, H, dtype=bf, device=dev)
    o = torch.empty_like(x)

    def exchange():
        cursor.zero_()  # the routing step's per-expert cursor, as moe_route leaves it
        C.ep_dispatch2(ctx.buf.peers, ctx.state, rank, ctx.cap, El, x, ids, counts, offs_g, cursor, emap, ctx.offs)
        C.ep_combine2(ctx.buf.peers, ctx.state, rank, ctx.cap, El, ctx.offs, y, emap, wts, None, o)
    us = _time(exchange, iters)
    out.append(_line("ep_dispatch_combine", "fused", us, 0, 2 * T * K * H * 2, nvl, world))
    from ..ops import check_status

    check_status(dev)
    if world > 1:
        nccl = NcclEPMoE(cfg, TorchBackend())
        us = _time(lambda: nccl(x, mo), max(3, iters // 10), warmup=2, graph=False)
        out.append(_line("ep_moe_layer", "nccl_baseline", us, flops, hbm, nvl, world))
    return out


def case_tp(iters, rank, world, dev, tokens=64):
    from ..parallel.symm import nvls_supported
    from ..parallel.tp import FusedTP, NcclTP, NvlsTP, padded_tokens

    H, Hq, Hkv, D, I = 4096, 32, 8, 128, 12288
    T = padded_tokens(tokens, world)
    pr = T // world
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(200 + rank)
    nq = (Hq + 2 * Hkv) * D // world
    w_qkv = (torch.randn(nq, H, device=dev, generator=g) * 0.02).to(bf)
    w_o = (torch.randn(H, Hq * D // world, device=dev, generator=g) * 0.02).to(bf)
    w_gu = (torch.randn(2 * I // world, H, device=dev, generator=g) * 0.02).to(bf)
    w_dn = (torch.randn(H, I // world, device=dev, generator=g) * 0.02).to(bf)
    nw = torch.ones(H, device=dev, dtype=bf)
    resid = torch.randn(pr, H, device=dev, generator=g).to(bf)
    attn = torch.randn(T, Hq * D // world, device=dev, generator=g).to(bf)
    flops = 2 * T * H * (nq + Hq * D // world + 2 * I // world) + 2 * T * (I // world) * H
    hbm = (w_qkv.numel() + w_o.numel() + w_gu.numel() + w_dn.numel()) * 2
    # two all-gathers (this shard to every peer) and two reduce-scatters (partials of the peers' rows)
    nvl = 2 * pr * H * 2 * (world - 1) + 2 * (T - pr) * H * 2
    out = []
    # fused = P2P flavour; +cluster: decode-sized gathered GEMMs as cluster launches (MB_TP_CLUSTER=1);
    # nvls = multimem reduce + multicast stores (where every rank's device has NVLink multicast)
    impls = [("fused", FusedTP(H, T))]
    if T <= 128:
        impls.append(("fused+cluster", impls[0][1]))
    if world > 1 and nvls_supported():
        nv = NvlsTP(H, T)
        impls.append(("nvls", nv))
        if T <= 128:
            impls.append(("nvls+cluster", nv))
    if world > 1:
        impls.append(("nccl_baseline", NcclTP(H, T)))
    for impl, comm in impls:
        os.environ["MB_TP_CLUSTER"] = "1" if impl.endswith("+cluster") else "0"
        def layer():
            comm.ag_gemm(w_qkv, T)
            comm.gemm_rs(attn, w_o)
            comm.publish(resid, nw, 1e-6, partials=True)
            h = comm.ag_gemm(w_gu, T, swiglu=True)
            comm.gemm_rs(h, w_dn)
            comm.publish(resid, nw, 1e-6, partials=True)
        comm.publish(resid, nw, 1e-6, partials=False)
        fused = impl != "nccl_baseline"
        us = _time(layer, iters if fused else max(5, iters // 5), graph=fused)
        out.append(_line("tp_layer_boundaries", impl, us, flops, hbm, nvl, world, {"tokens": T}))
    from ..ops import check_status

    check_status(dev)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="ep,tp")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--tp-tokens", default="64", help="comma-separated token counts of the TP case")
    ap.add_argument("--profile", action="store_true", help="per-kernel table of each timed path (rank 0)")
    a = ap.parse_args(argv)
    PROFILE["on"] = a.profile
    from ..parallel import dist as mdist

    info = mdist.init()
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    for c in a.case.split(","):
        if c == "tp":
            recs = [r for n in a.tp_tokens.split(",") for r in case_tp(a.iters, info.rank, info.world, dev, int(n))]
        else:
            recs = case_ep(a.iters, info.rank, info.world, dev)
        if info.rank == 0:
            for r in recs:
                print(json.dumps(r), flush=True)
            for t in PROFILE["tables"]:
                print(t, flush=True)
        PROFILE["tables"].clear()
    mdist.barrier()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
