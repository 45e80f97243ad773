"""Sanitizer build of the C++ CPU backend (AddressSanitizer + UBSan).

The reference builds its C library with ``-Wall -Wextra`` only
(``build_ops.py:26``) and its own tests sort results to hide OpenMP races
(``tests/test_moe_dispatch.py:39-49``); its CPU attention overruns the heap on
GQA shapes (``src/inference_pio/plugins/cpu/c_src/tensor_ops.c:384-415``).

``build(kind)`` compiles ``csrc/cpu`` + ``csrc/io`` with ``-fsanitize=<kind>``
into a separate extension (``_cpu_<kind>``) in a scratch directory.
``python -m mod_b200.utils.sanitize <build_dir> [kind]`` builds it and runs the CPU
backend's workloads -- dense, MoE and hybrid DeltaNet generation, the
safetensors reader on a valid and on truncated files -- on that build, with
the sanitized module standing in for ``mod_b200._cpu``.  A sanitizer report
aborts the process with a non-zero exit code.  The sanitizer runtime must be
loaded first, so the runner is started with ``LD_PRELOAD`` set to it
(``runtime_library(kind)``); ``run(kind)`` does all of this in a subprocess.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from typing import Optional

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
# ThreadSanitizer is left out: libgomp is not instrumented, so every OpenMP barrier would be reported
_RUNTIME = {"address": "libasan.so"}


def runtime_library(kind: str) -> str:
    out = subprocess.run(["gcc", f"-print-file-name={_RUNTIME[kind]}"], capture_output=True, text=True, check=True)
    return out.stdout.strip()


def _libstdcxx() -> str:
    out = subprocess.run(["g++", "-print-file-name=libstdc++.so.6"], capture_output=True, text=True, check=True)
    return out.stdout.strip()


def build(kind: str, build_dir: str, verbose: bool = False):
    from torch.utils.cpp_extension import load

    flags = {"address": ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"]}[kind]
    srcs = sorted(glob.glob(os.path.join(ROOT, "csrc", "cpu", "*.cc"))) + \
        sorted(glob.glob(os.path.join(ROOT, "csrc", "io", "*.cc")))
    os.makedirs(build_dir, exist_ok=True)
    # the system driver knows where the sanitizer runtimes live; a bare wrapper on CXX may not
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
    return load(name=f"_cpu_{kind}", sources=srcs, build_directory=build_dir, verbose=verbose,
                extra_include_paths=[os.path.join(ROOT, "csrc", "cpu"), os.path.join(ROOT, "csrc", "io")],
                extra_cflags=["-O1", "-g", "-std=c++17", "-fopenmp", "-march=x86-64-v3",
                              "-fno-omit-frame-pointer"] + flags,
                extra_ldflags=["-fopenmp"] + flags)


def _workloads(tmp: str) -> None:
    import torch

    from ..config import get_preset
    from ..engine.llm_engine import LLMEngine
    from ..engine.sequence import SamplingParams
    from ..io import safetensors as st
    from ..models.weights import random_weights

    prompts = [[1, 2, 3, 4, 5, 6, 7], [9, 8, 7], [11] * 20]
    for name in ("tiny-dense", "tiny-moe", "tiny-next"):
        cfg = get_preset(name)
        w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=0)
        got = LLMEngine(cfg, weights=w, backend="cpu", device="cpu", max_batch=4,
                        max_model_len=64).generate(prompts, SamplingParams(max_new_tokens=6))
        ref = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=4,
                        max_model_len=64).generate(prompts, SamplingParams(max_new_tokens=6))
        same = sum(a == b for a, b in zip(got, ref))
        print(f"{name}: {same}/{len(ref)} sequences token-identical to the torch fp32 path", flush=True)
    p = os.path.join(tmp, "w.safetensors")
    t = {"a": torch.arange(12, dtype=torch.float32).reshape(3, 4), "b": torch.ones(5, dtype=torch.bfloat16)}
    st.save_file(p, t)
    f = st.open_file(p)
    assert torch.equal(f.get("a"), t["a"]) and torch.equal(f.get_slice("a", 0, 1, 3), t["a"][1:2])
    raw = open(p, "rb").read()
    for cut in (4, 12, len(raw) // 2, len(raw) - 1):
        q = os.path.join(tmp, f"cut{cut}.safetensors")
        with open(q, "wb") as fh:
            fh.write(raw[:cut])
        try:
            st.open_file(q).get("b")
        except Exception:
            pass
        else:
            raise AssertionError(f"truncated file ({cut} bytes) was accepted")
    print("safetensors: valid file read, truncated files rejected", flush=True)


def run(kind: str = "address", build_dir: Optional[str] = None, timeout: float = 1200.0) -> str:
    """Build the sanitized backend and run the workloads in a child process; returns its output."""
    build_dir = build_dir or os.path.join(ROOT, "_build", f"sanitize_{kind}")
    env = dict(os.environ)
    # libstdc++ right after the runtime, so the runtime's exception interceptor finds the real __cxa_throw
    # (the extension reports bad input, e.g. a truncated safetensors file, with C++ exceptions)
    env["LD_PRELOAD"] = runtime_library(kind) + " " + _libstdcxx()
    env["ASAN_OPTIONS"] = "detect_leaks=0:abort_on_error=1"
    env["UBSAN_OPTIONS"] = "print_stacktrace=1:halt_on_error=1"
    env["OMP_NUM_THREADS"] = env.get("OMP_NUM_THREADS", "4")
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    p = subprocess.run([sys.executable, "-m", "mod_b200.utils.sanitize", build_dir, kind], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=timeout)
    out = p.stdout + p.stderr
    if p.returncode != 0:
        raise RuntimeError(f"sanitized CPU backend run failed (rc={p.returncode}):\n{out[-6000:]}")
    return out


def _main(build_dir: str, kind: str) -> None:
    import tempfile

    import torch  # noqa: F401  (libc10 first)

    # built (and imported) here, in the process that has the sanitizer runtime preloaded
    mod = build(kind, build_dir)
    sys.modules["mod_b200._cpu"] = mod  # the CPU backend and safetensors reader import this name
    with tempfile.TemporaryDirectory() as tmp:
        _workloads(tmp)
    print("sanitizer run clean", flush=True)


if __name__ == "__main__":
    _main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "address")
