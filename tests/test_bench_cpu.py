"""Benchmark entry points that run without a GPU: the config #1 CPU benchmark
(short run) and bench.py's reference arm, whose JSON lines the tooling reads."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _json_line(out: str) -> dict:
    return json.loads([l for l in out.splitlines() if l.startswith("{")][-1])


def test_cpu_config1_short_run():
    r = subprocess.run([sys.executable, "-m", "mod_b200.bench.cpu_config1", "--prompt-len", "16", "--new-tokens", "4",
                        "--threads", "4"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    d = _json_line(r.stdout)
    assert d["backend"] == "cpu" and d["ttft_s"] > 0 and d["decode_tok_s"] > 0


def test_bench_reference_arm_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    d = _json_line(r.stdout)
    assert d["impl"] == "reference" and ("unavailable" in d or "value" in d)
