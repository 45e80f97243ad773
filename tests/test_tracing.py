"""Tracing helpers on CPU: NVTX ranges are inert without a GPU, torch.profiler
traces export, DeviceTimer falls back to host timing, the decoder runs with
per-layer ranges enabled."""
import json

import torch

from mod_b200.utils import tracing


def test_nvtx_range_toggle():
    tracing.enable_nvtx(True)
    try:
        with tracing.nvtx_range("outer"):
            with tracing.nvtx_range("inner"):
                x = torch.ones(3) * 2
    finally:
        tracing.enable_nvtx(False)
    assert float(x.sum()) == 6.0
    with tracing.nvtx_range("off"):
        pass


def test_trace_exports_chrome_json(tmp_path):
    p = tmp_path / "t" / "trace.json"
    with tracing.trace(str(p), cuda=False):
        torch.mm(torch.randn(32, 32), torch.randn(32, 32))
    d = json.loads(p.read_text())
    names = {e.get("name", "") for e in d["traceEvents"]}
    assert any("mm" in n for n in names)


def test_device_timer_cpu():
    t = tracing.DeviceTimer(device="cpu")
    for _ in range(3):
        with t.region():
            torch.randn(64, 64).sum()
    assert t.count == 3 and t.result_ms() > 0.0


def test_decoder_forward_with_nvtx_ranges():
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.engine.sequence import SamplingParams

    eng = LLMEngine(get_preset("tiny-dense"), backend="torch", device="cpu", max_batch=2, max_model_len=64)
    ref = eng.generate([[1, 2, 3]], SamplingParams(max_new_tokens=3))
    tracing.enable_nvtx(True)
    try:
        out = eng.generate([[1, 2, 3]], SamplingParams(max_new_tokens=3))
    finally:
        tracing.enable_nvtx(False)
    assert out == ref
