"""Command line: ``python -m mod_b200 <command>``.

Commands mirror the reference CLI (``pio/__main__.py:266-343``: list, run,
chat, info, config, benchmark, check, init, clean), which fails at import in
the reference because three of its modules are missing:

  list                 plugins and their manifests
  info MODEL           architecture / parameter counts
  run MODEL --prompt   one generation
  chat MODEL           interactive loop (ChatML, thinking mode on/off)
  config list|view     presets, profiles, a preset's fields
  benchmark            the decode benchmark (bench.py) or a quick synthetic run
  check                environment: devices, peer access, extensions
  init DIR             writes a runtime config template
  clean                removes build outputs and caches
  plan MODEL --gpus N  parallel degrees, per-GPU weight and KV memory
  serve MODEL          HTTP completions server (OpenAI-style route, streaming)
  tune MODEL           measured GEMM launch configurations (JSON cache)
  trace MODEL          torch.profiler trace of a short generation
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import shutil
import subprocess
import sys
import time
from typing import List, Optional

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _pm():
    from ..api import get_plugin_manager

    return get_plugin_manager()


def _opts(args) -> dict:
    o = {}
    for kv in args.set or []:
        k, _, v = kv.partition("=")
        try:
            v = json.loads(v)
        except json.JSONDecodeError:
            pass
        o[k] = v
    if getattr(args, "device", None):
        o["device"] = args.device
    if getattr(args, "backend", None):
        o["backend"] = args.backend
    off = getattr(args, "offload_layers", None)
    if off:  # hybrid CPU/GPU execution: "auto" (planner) or a layer count
        o["offload_layers" if off != "auto" else "offload"] = int(off) if off != "auto" else True
    return o


def cmd_list(args) -> int:
    for m in _pm().list_plugins():
        print(f"{m['name']:28s} {m.get('model_architecture', ''):50s} {','.join(m.get('supported_modalities') or [])}")
    return 0


def cmd_info(args) -> int:
    from ..config import get_preset

    pm = _pm()
    name = pm.resolve(args.model)
    m = pm.manifests.get(name, {})
    cfg = get_preset(m.get("preset", args.model))
    text = getattr(cfg, "text", cfg)
    info = {"name": name, "preset": m.get("preset"), "parameters": text.num_params(),
            "active_parameters": text.active_params(), "config": dataclasses.asdict(cfg)}
    print(json.dumps(info, indent=2, default=str))
    return 0


def cmd_run(args) -> int:
    pm = _pm()
    if not pm.activate_plugin(args.model, **_opts(args)):
        print("initialisation failed", file=sys.stderr)
        return 1
    p = pm.get_plugin(args.model)
    t0 = time.perf_counter()
    out = p.generate_text(args.prompt, max_new_tokens=args.max_new_tokens, temperature=args.temperature)
    dt = time.perf_counter() - t0
    print(out)
    print(f"[{args.max_new_tokens} tokens in {dt:.2f} s]", file=sys.stderr)
    return 0


def cmd_chat(args) -> int:
    from ..io.prompts import apply_chat_template, format_history, strip_thinking

    pm = _pm()
    if not pm.activate_plugin(args.model, **_opts(args)):
        return 1
    p = pm.get_plugin(args.model)
    history: List[dict] = []
    print("type /exit to quit")
    for line in sys.stdin:
        line = line.strip()
        if line in ("/exit", "/quit"):
            break
        history.append({"role": "user", "content": line})
        text = apply_chat_template(p.tokenizer, format_history(history), enable_thinking=args.thinking)
        reply = p.generate_text(text, max_new_tokens=args.max_new_tokens)
        history.append({"role": "assistant", "content": reply})
        print(strip_thinking(reply))
    return 0


def cmd_config(args) -> int:
    from ..config import PRESETS, get_preset
    from ..config.runtime import PROFILES

    if args.action == "list":
        print("presets:", ", ".join(sorted(PRESETS)))
        print("profiles:", ", ".join(sorted(PROFILES)))
        base = os.path.join(ROOT, "mod_b200", "config", "baselines")
        print("baseline configs:", ", ".join(sorted(os.listdir(base))))
    else:
        print(json.dumps(dataclasses.asdict(get_preset(args.name)), indent=2, default=str))
    return 0


def cmd_benchmark(args) -> int:
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--steps", str(args.steps), "--warmup", str(args.warmup),
           "--impl", args.impl]
    if args.gpus > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}",
               "--master-addr=127.0.0.1", "--master-port=29533"] + cmd[1:] + ["--gpus", str(args.gpus)]
    return subprocess.call(cmd)


def cmd_check(args) -> int:
    from ..api.backends import probe_system
    from ..ops import extension_available

    info = probe_system()
    info["extension_cuda"] = extension_available()
    try:
        import mod_b200._cpu  # noqa: F401

        info["extension_cpu"] = True
    except ImportError:
        info["extension_cpu"] = False
    print(json.dumps(info, indent=2))
    return 0 if info["extension_cpu"] else 1


def cmd_init(args) -> int:
    from ..config.runtime import RuntimeConfig, save

    os.makedirs(args.dir, exist_ok=True)
    path = os.path.join(args.dir, "runtime.yaml")
    save(RuntimeConfig(), path)
    print(f"wrote {path}")
    return 0


def cmd_clean(args) -> int:
    for d in ("build", "_build"):
        p = os.path.join(ROOT, d)
        if os.path.isdir(p):
            shutil.rmtree(p)
            print(f"removed {p}")
    for dirpath, dirnames, _ in os.walk(ROOT):
        for d in list(dirnames):
            if d in ("__pycache__", ".pytest_cache"):
                shutil.rmtree(os.path.join(dirpath, d), ignore_errors=True)
                dirnames.remove(d)
    return 0


def cmd_tune(args) -> int:
    import torch

    from ..config import get_preset
    from ..ops import autotune

    if not torch.cuda.is_available():
        print("tune: needs a GPU (the cache holds measured kernel times)")
        return 1
    cfg = get_preset(args.model)
    cache = autotune.TuneCache(args.out)
    for shape in autotune.model_linear_shapes(cfg, args.tokens):
        e = autotune.tune_linear(*shape, cache, reps=args.reps)
        print(f"T={shape[0]:5d} N={shape[1]:6d} K={shape[2]:6d}  splits={e['splits']:2d} orient={e['orient']}  "
              f"{e['us']:.1f} us")
    cache.save()
    print(f"wrote {args.out}; use it with MB_TUNE_CACHE={args.out}")
    return 0


def cmd_trace(args) -> int:
    from ..config import get_preset
    from ..engine.llm_engine import LLMEngine
    from ..engine.sequence import SamplingParams
    from ..utils import tracing

    eng = LLMEngine(get_preset(args.model), backend=args.backend, device=args.device,
                    max_batch=args.batch, max_model_len=args.prompt_len + args.max_new_tokens + 16)
    prompts = [[1 + (i + j) % 500 for j in range(args.prompt_len)] for i in range(args.batch)]
    eng.generate(prompts, SamplingParams(max_new_tokens=2))  # warm-up (graph capture, first launches)
    tracing.enable_nvtx(True)
    with tracing.trace(args.out):
        eng.generate(prompts, SamplingParams(max_new_tokens=args.max_new_tokens))
    print(f"wrote {args.out}")
    return 0


def cmd_serve(args) -> int:
    """One process: the server over its engine.  Under ``torch.distributed.run`` (one process
    per GPU): every rank builds its part of the model (``--set tp=N`` for tensor parallelism;
    MoE models are expert parallel), rank 0 serves HTTP through a front-end that broadcasts the
    requests, and the other ranks run the same loop without a server."""
    import os

    from ..api.server import serve

    world = int(os.environ.get("WORLD_SIZE", "1"))
    opts = _opts(args)
    if world > 1:
        from ..parallel import dist as mdist

        info = mdist.init()
        if opts.get("device", "cuda") != "cpu":
            opts["device"] = f"cuda:{info.local_rank}"
    pm = _pm()
    if not pm.activate_plugin(args.model, **opts):
        print("initialisation failed", file=sys.stderr)
        return 1
    p = pm.get_plugin(args.model)
    if world == 1:
        serve(p.engine, p.tokenizer, args.model, host=args.host, port=args.port)
        return 0
    from ..api.dist_front import DistributedFrontEnd

    eng = p.engine
    mode = "tp" if eng.tensor_parallel else ("ep" if eng.expert_parallel else "dp")
    front = DistributedFrontEnd(eng, mode)
    if front.rank == 0:
        serve(front, p.tokenizer, args.model, host=args.host, port=args.port)
    else:
        front.run()
    return 0


def cmd_plan(args) -> int:
    from ..config import get_preset
    from ..parallel.planner import plan

    p = plan(get_preset(args.model), args.gpus, hbm_bytes=int(args.hbm_gb * 1e9), int8=args.int8,
             attn=getattr(args, "attn", "dp"))
    print(json.dumps(p.as_dict(), indent=1))
    return 0 if p.fits else 2


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="mod_b200", description="B200-native LLM/VLM inference engine")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--version", action="version", version="mod_b200 0.1.0")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("list").set_defaults(fn=cmd_list)
    p = sub.add_parser("info")
    p.add_argument("model")
    p.set_defaults(fn=cmd_info)
    for name, fn in (("run", cmd_run), ("chat", cmd_chat)):
        p = sub.add_parser(name)
        p.add_argument("model")
        p.add_argument("--device")
        p.add_argument("--backend", choices=["native", "torch", "cpu"])
        p.add_argument("--max-new-tokens", type=int, default=64)
        p.add_argument("--set", nargs="*", help="config overrides key=value")
        p.add_argument("--offload-layers", help="stream the last N layers from pinned host memory ('auto': planner)")
        if name == "run":
            p.add_argument("--prompt", required=True)
            p.add_argument("--temperature", type=float, default=0.0)
        else:
            p.add_argument("--thinking", action="store_true")
        p.set_defaults(fn=fn)
    p = sub.add_parser("config")
    p.add_argument("action", choices=["list", "view"])
    p.add_argument("name", nargs="?", default="qwen3-0.6b")
    p.set_defaults(fn=cmd_config)
    p = sub.add_parser("benchmark")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=32)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="native", choices=["native", "baseline", "reference"])
    p.set_defaults(fn=cmd_benchmark)
    sub.add_parser("check").set_defaults(fn=cmd_check)
    p = sub.add_parser("init")
    p.add_argument("dir")
    p.set_defaults(fn=cmd_init)
    sub.add_parser("clean").set_defaults(fn=cmd_clean)
    p = sub.add_parser("plan", help="parallel degrees and per-GPU memory for a model on N GPUs")
    p.add_argument("model")
    p.add_argument("--gpus", type=int, default=8)
    p.add_argument("--hbm-gb", type=float, default=180.0)
    p.add_argument("--int8", action="store_true")
    p.add_argument("--attn", default="dp", choices=["dp", "tp"], help="MoE models: attention data- or tensor-parallel")
    p.set_defaults(fn=cmd_plan)
    p = sub.add_parser("serve", help="HTTP completions server (one engine, or one per GPU under torchrun)")
    p.add_argument("model")
    p.add_argument("--device")
    p.add_argument("--backend", choices=["native", "torch", "cpu"])
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--set", nargs="*", help="config overrides key=value")
    p.set_defaults(fn=cmd_serve)
    p = sub.add_parser("tune", help="measure GEMM launch configurations for a model's shapes")
    p.add_argument("model")
    p.add_argument("--tokens", type=int, nargs="+", default=[1, 8, 32, 64, 128, 256])
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--out", default="tune_cache.json")
    p.set_defaults(fn=cmd_tune)
    p = sub.add_parser("trace", help="torch.profiler trace (Chrome JSON) of a short generation")
    p.add_argument("model")
    p.add_argument("--backend", default="native", choices=["native", "torch", "cpu"])
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--prompt-len", type=int, default=32)
    p.add_argument("--max-new-tokens", type=int, default=8)
    p.add_argument("--out", default="trace.json")
    p.set_defaults(fn=cmd_trace)
    return ap


def main(argv: Optional[List[str]] = None) -> int:
    from ..utils.logging import setup_logging

    args = build_parser().parse_args(argv)
    setup_logging(debug=args.debug)
    return args.fn(args)
