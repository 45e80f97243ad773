"""BASELINE config #1: Qwen3-0.6B-shaped dense decoder on the C++ CPU backend.

    python -m mod_b200.bench.cpu_config1 [--threads 8] [--new-tokens 128]

fp32, random N(0, 0.02) weights from seed 0, batch 1, a 128-token prompt of
uniform-random ids, greedy decode.  Reports TTFT (prefill + first token) and
decode tokens/s through the public engine API.  The reference's CPU C backend
was measured at 9.12 s TTFT and 10.78 tok/s on an 8-vCPU Xeon, on the MHA
variant of this shape (its GQA path aborts).
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--backend", default="cpu", choices=["cpu", "torch"])
    ap.add_argument("--weight-dtype", default="fp32", choices=["fp32", "bf16", "int8"],
                    help="bf16 / int8 (per-channel scales): projection weights stored narrower, fp32 math; "
                         "config #1 itself is fp32")
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..engine import SamplingParams
    from ..engine.llm_engine import LLMEngine
    from ..models.backend import CpuBackend
    from ..models.weights import random_weights

    if a.threads:
        torch.set_num_threads(a.threads)
    cfg = get_preset("qwen3-0.6b")
    t0 = time.perf_counter()
    w = random_weights(cfg, device="cpu", dtype=torch.bfloat16 if a.weight_dtype == "bf16" else torch.float32,
                       seed=0)
    if a.weight_dtype == "int8":
        from ..ops.quant import quantize_model

        quantize_model(w)
        # embedding / LM head stay out of int8 (as on the GPU path); store them bf16 here
        tied = w.lm_head is w.embed
        w.embed = w.embed.bfloat16()
        w.lm_head = w.embed if tied else w.lm_head.bfloat16()
    init_s = time.perf_counter() - t0
    eng = LLMEngine(cfg, weights=w, backend=a.backend, device="cpu", max_batch=1,
                    max_model_len=a.prompt_len + a.new_tokens + 16)
    if a.backend == "cpu" and a.threads:
        eng.backend.C.set_num_threads(a.threads)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist()
    rid = eng.add_request(prompt, SamplingParams(max_new_tokens=a.new_tokens, ignore_eos=True))
    t0 = time.perf_counter()
    eng.step()                                   # prefill + first token
    ttft = time.perf_counter() - t0
    t1 = time.perf_counter()
    n = 0
    while eng.has_unfinished():
        eng.step()
        n += 1
    dec = time.perf_counter() - t1
    label = {"fp32": "fp32", "bf16": "bf16 weights, fp32 math",
             "int8": "int8 projections + bf16 embedding / LM head, fp32 math"}[a.weight_dtype]
    print(json.dumps({"config": f"qwen3-0.6b cpu {label} (16/8 GQA, head_dim 128, QK-norm)", "backend": a.backend,
                      "threads": a.threads or os.cpu_count(), "prompt_len": a.prompt_len, "ttft_s": round(ttft, 3),
                      "decode_tok_s": round(n / dec, 2), "decode_ms_per_token": round(dec / n * 1000, 2),
                      "weights_init_s": round(init_s, 1),
                      "reference": {"ttft_s": 9.12, "decode_tok_s": 10.78, "note": "reference MHA variant, 8 vCPU"}}))


if __name__ == "__main__":
    main()
