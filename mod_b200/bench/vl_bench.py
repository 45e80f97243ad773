"""BASELINE config #4: Qwen3-VL-style model (ViT patch 16, 24 x 1024, 2x2 merge;
28-layer 2048-wide decoder), bf16, random-init, batch 16 of 448x448 images
(pixels uniform in [0, 1], mean/std normalised on the GPU) + 64 text tokens.

    python -m torch.distributed.run --nproc-per-node N -m mod_b200.bench.vl_bench [--impl native|baseline]

N = 1: single-GPU ``VLModel``.  N > 1: ``TPVLModel`` - TP decoder, vision
encoder data-parallel over the images, merger output delivered to the
owners of the token rows (native: fused GEMM + P2P exchange; baseline: NCCL
all-gather + cuBLAS).  Reports the batch prefill time (images + text, all
requests arriving at once), p50 TTFT, and decode tokens/s over graph replays
(device time, max over ranks).
"""
from __future__ import annotations

import argparse
import json
import time

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", default="native", choices=["native", "baseline"])
    ap.add_argument("--comm", default="auto", choices=["p2p", "nvls", "auto"],
                    help="layer-boundary flavour of the native path")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--text-len", type=int, default=64)
    ap.add_argument("--image-size", type=int, default=448)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..engine import SamplingParams
    from ..engine.llm_engine import LLMEngine
    from ..models.backend import make_backend
    from ..models.tp_decoder import shard_weights
    from ..models.vl import TPVLModel, VLModel, random_vl_weights
    from ..parallel import dist as mdist
    from ..parallel.tp import FusedVisionExchange, NcclVisionExchange, make_tp_comm

    info = mdist.init()
    world, rank = info.world, info.rank
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    cfg = get_preset("qwen3-vl")
    backend = "native" if a.impl == "native" else "torch"
    be = make_backend(backend)
    tw, vw = random_vl_weights(cfg, device=dev, seed=0)
    p, m = cfg.vision.patch_size, cfg.vision.spatial_merge_size
    per_img = (a.image_size // p) ** 2 // (m * m)
    max_tokens = a.batch * (per_img + a.text_len)
    if world > 1:
        H = cfg.text.hidden_size
        comm = make_tp_comm(a.comm if backend == "native" else "nccl", H, max_tokens)
        vx = FusedVisionExchange(H, max_tokens) if backend == "native" else NcclVisionExchange(be)
        model = TPVLModel(cfg, shard_weights(cfg.text, tw, rank, world), vw, be, comm, world, vx,
                          image_size=a.image_size)
        tw = None
    else:
        model = VLModel(cfg, tw, vw, be, image_size=a.image_size)
    eng = LLMEngine(cfg.text, model=model, backend=backend, device=dev, max_batch=a.batch,
                    max_model_len=per_img + a.text_len + a.warmup + 3 * a.steps + 16, max_prefill_tokens=max_tokens,
                    tensor_parallel=world > 1)
    g = torch.Generator().manual_seed(11)
    imgs = [torch.rand(3, a.image_size, a.image_size, generator=g).to(dev, torch.bfloat16) for _ in range(a.batch)]
    texts = [torch.randint(0, cfg.text.vocab_size, (a.text_len,), generator=g).tolist() for _ in range(a.batch)]
    params = SamplingParams(max_new_tokens=a.warmup + 3 * a.steps + 8, ignore_eos=True)
    mdist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ids = [eng.add_request(model.prompt_with_image(t), params, images=im) for t, im in zip(texts, imgs)]
    while any(eng.seqs[i].t_first_token is None for i in ids):
        eng.step()
    torch.cuda.synchronize()
    prefill_s = mdist.max_over_ranks(time.perf_counter() - t0, dev)
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
    if backend == "native":
        from ..ops import check_status

        check_status(dev)
    if rank == 0:
        print(json.dumps({"config": f"qwen3-vl TP={world}", "impl": a.impl, "batch": a.batch,
                          "visual_tokens_per_image": per_img, "text_len": a.text_len,
                          "prefill_s": round(prefill_s, 4), "ttft_p50_s": round(p50, 4),
                          "decode_ms_per_step": round(ms, 3), "decode_tok_s": round(a.batch / ms * 1000, 1),
                          "timed": "graph replay" if B is not None else "eager engine steps"}), flush=True)
    mdist.barrier()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
