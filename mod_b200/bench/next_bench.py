"""BASELINE config #5: Qwen3-Next-style hybrid (3 gated-DeltaNet : 1 gated
attention layers, 512 experts top-10 + shared expert), batch 4.

    python -m mod_b200.bench.next_bench [--prompt-len 32768] [--steps 16] [--quant int8]

Random-init N(0, 0.02) weights (int8 weight-only per-channel by default, made
layer by layer so the bf16 model is never resident), uniform-random prompt
ids.  Reports the prefill wall time of the batch (all prompts arrive at once,
chunked by --prefill-tokens), and decode tokens/s: device-timed CUDA-graph
replays (CUDA events) and end to end through ``LLMEngine.step()``.  Under
``torch.distributed.run`` with N processes: the TP/EP form (``--attn tp``, the
default: DeltaNet and attention heads split over the ranks, experts expert-parallel),
or expert parallelism with
data-parallel attention (sequence i on rank i % N; ranks without a sequence take
part in the MoE exchanges with padding rows), times as the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import time

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt-len", type=int, default=32768)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--quant", default="int8", choices=["int8", "none"])
    ap.add_argument("--impl", default="native", choices=["native", "baseline"],
                    help="baseline: PyTorch + cuBLAS + NCCL (library exchange and GEMMs, same engine)")
    ap.add_argument("--prefill-tokens", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (smoke runs only)")
    ap.add_argument("--attn", default="tp", choices=["tp", "dp"],
                    help="N > 1: heads tensor-parallel (every rank all sequences) or attention data-parallel "
                         "(sequence i on rank i %% N); experts expert-parallel either way")
    a = ap.parse_args(argv)
    import os

    from ..config import get_preset
    from ..engine import SamplingParams
    from ..engine.llm_engine import LLMEngine
    from ..models.weights import random_weights
    from ..ops import check_status
    from ..parallel import dist as mdist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = 0
    if world > 1:  # expert parallel with data-parallel attention: sequence i on rank i % world
        info = mdist.init()
        rank = info.rank
        dev = torch.device("cuda", info.local_rank)
    else:
        dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = get_preset("qwen3-next")
    if a.layers:
        cfg.num_hidden_layers = a.layers
        cfg.layer_types = cfg.layer_types[:a.layers]
    tp_attn = world > 1 and a.attn == "tp"
    backend = "native" if a.impl == "native" else "torch"
    if backend == "torch" and a.quant != "none":
        raise SystemExit("the library baseline runs bf16 weights: pass --quant none")
    if tp_attn and a.quant != "none":
        raise SystemExit("the tensor-parallel form runs bf16 weights: pass --quant none (or --attn dp for int8)")
    per_rank = a.batch if tp_attn else max(1, -(-a.batch // world))
    max_len = a.prompt_len + a.warmup + 3 * a.steps + 16
    t0 = time.perf_counter()
    if world == 1:
        w = random_weights(cfg, device=dev, seed=0, quantize=None if a.quant == "none" else a.quant)
        torch.cuda.synchronize()
        init_s = time.perf_counter() - t0
        eng = LLMEngine(cfg, weights=w, backend=backend, device=dev, max_batch=a.batch, max_model_len=max_len,
                        max_prefill_tokens=a.prefill_tokens)
    else:  # this rank's experts (bf16 under expert parallelism), int8 projections with --quant int8
        eng = LLMEngine(cfg, backend=backend, device=dev, max_batch=per_rank, max_model_len=max_len,
                        max_prefill_tokens=a.prefill_tokens, expert_parallel=not tp_attn,
                        tensor_parallel=tp_attn, seed=0,
                        quantization=None if a.quant == "none" else a.quant)
        torch.cuda.synchronize()
        init_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist() for _ in range(a.batch)]
    mine = prompts if tp_attn else prompts[rank::world]
    params = SamplingParams(max_new_tokens=a.warmup + 3 * a.steps + 8, ignore_eos=True)

    def pending_anywhere(ids) -> bool:  # every rank must agree on when to stop stepping
        p = any(eng.seqs[i].t_first_token is None for i in ids)
        return bool(mdist.max_over_ranks(float(p), dev)) if world > 1 else p

    mdist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ids = [eng.add_request(p, params) for p in mine]
    while pending_anywhere(ids):
        eng.step()
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    if world > 1:
        prefill_s = mdist.max_over_ranks(prefill_s, dev)
    for _ in range(a.warmup):
        eng.step()
    r = eng.runner
    # the captured decode step of this rank (its batch's bucket, or the padding-row graph of an idle rank);
    # every rank's graph holds the same MoE exchanges, so the ranks replay them together
    B = None
    if r.graphs:
        B = r.buckets[r.bucket_index(len(mine))] if mine else r.buckets[0]
        B = B if B in r.graphs else None
    step = (lambda: r.graphs[B].replay()) if B is not None else eng.step
    mdist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(a.steps):
        step()
    e.record()
    torch.cuda.synchronize()
    dev_ms = s.elapsed_time(e) / a.steps
    mdist.barrier()
    t1 = time.perf_counter()
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t1) * 1000 / a.steps
    if world > 1:
        dev_ms = mdist.max_over_ranks(dev_ms, dev)
        e2e_ms = mdist.max_over_ranks(e2e_ms, dev)
    check_status(dev)
    if rank == 0:
        print(json.dumps({"config": "qwen3-next hybrid (3 DeltaNet : 1 gated attention, 512 experts top-10 + shared)",
                          "impl": a.impl, "quant": a.quant, "batch": a.batch, "prompt_len": a.prompt_len,
                          "layers": cfg.num_hidden_layers, "n_gpus": world,
                          "parallelism": f"ep{world}+{a.attn}_attn{world}" if world > 1 else "single",
                          "weights_init_s": round(init_s, 1), "prefill_s": round(prefill_s, 3),
                          "prefill_tok_s": round(a.batch * a.prompt_len / prefill_s, 1),
                          "decode_ms_per_step": round(dev_ms, 3), "decode_tok_s": round(a.batch / dev_ms * 1000, 1),
                          "e2e_decode_tok_s": round(a.batch / e2e_ms * 1000, 1),
                          "timed": "graph replay" if B is not None else "eager engine steps",
                          "invalid": "layer count overridden" if a.layers else None}), flush=True)
    if world > 1:
        mdist.barrier()


if __name__ == "__main__":
    main()
