"""BASELINE config #2: Qwen3-8B-shaped dense decoder, tensor parallel.

    torchrun --nproc-per-node N -m mod_b200.bench.tp_bench [--impl native|baseline]

bf16, random-init N(0, 0.02), paged KV (block 16), batch 64, prompts of 1024
uniform-random ids.  Reports p50 TTFT of the batch (all prompts arrive at
once; prefill runs in chunks of --prefill-tokens) and decode tokens/s of the
whole job (device-timed CUDA-graph replays, max over ranks).  native = fused
NVLink all-gather->GEMM / GEMM->reduce-scatter; baseline = NCCL + cuBLAS.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", default="native", choices=["native", "baseline"])
    ap.add_argument("--comm", default="auto", choices=["p2p", "nvls", "auto"],
                    help="layer-boundary flavour of the native path")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--prefill-tokens", type=int, default=16384)
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--profile", action="store_true", help="print a per-kernel table of 3 decode steps (rank 0)")
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..engine import SamplingParams
    from ..engine.llm_engine import LLMEngine
    from ..parallel import dist as mdist

    info = mdist.init()
    world, rank = info.world, info.rank
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    cfg = get_preset(a.model)
    backend = "native" if a.impl == "native" else "torch"
    eng = LLMEngine(cfg, backend=backend, device=dev, max_batch=a.batch,
                    max_model_len=a.prompt_len + a.warmup + 3 * a.steps + 16, max_prefill_tokens=a.prefill_tokens,
                    tensor_parallel=world > 1, seed=0, tp_comm=a.comm)
    g = torch.Generator().manual_seed(1000)
    prompts = [torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist() for _ in range(a.batch)]
    params = SamplingParams(max_new_tokens=a.warmup + 3 * a.steps + 8, ignore_eos=True)
    mdist.barrier()
    torch.cuda.synchronize()
    ids = [eng.add_request(p, params) for p in prompts]
    while any(eng.seqs[i].t_first_token is None for i in ids):
        eng.step()
    torch.cuda.synchronize()
    ttfts = sorted(eng.seqs[i].ttft for i in ids)
    p50 = mdist.max_over_ranks(ttfts[len(ttfts) // 2], dev)
    for _ in range(a.warmup):
        eng.step()
    r = eng.runner
    B = max(r.graphs) if r.graphs else None
    step = (lambda: r.graphs[B].replay()) if B is not None else eng.step
    mdist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(a.steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = mdist.max_over_ranks(s.elapsed_time(e) / a.steps, dev)
    if a.profile:
        from .profile import kernel_table

        table = kernel_table(step, 3)
        if rank == 0:
            print(table)
    if backend == "native":
        from ..ops import check_status

        check_status(dev)
    if rank == 0:
        print(json.dumps({"config": f"{a.model} TP={world}", "impl": a.impl,
                          "comm": type(getattr(eng.model, "comm", None)).__name__, "batch": a.batch,
                          "prompt_len": a.prompt_len, "ttft_p50_s": round(p50, 4), "decode_ms_per_step": round(ms, 3),
                          "decode_tok_s": round(a.batch / ms * 1000, 1),
                          "timed": "graph replay" if B is not None else "eager engine steps"}), flush=True)
    mdist.barrier()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
