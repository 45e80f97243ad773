"""GEMM launch-configuration cache: JSON round trip and lookup on CPU; tuning
and tuned launches against a torch fp32 reference on the GPU."""
import pytest
import torch

from mod_b200.ops import autotune


def test_cache_roundtrip_and_lookup(tmp_path):
    p = str(tmp_path / "tune.json")
    c = autotune.TuneCache(p, device_name="B200-test")
    c.put((64, 4096, 2048), 4, 1, 12.5, {"s1o0": 30.0, "s4o1": 12.5})
    c.save()
    c2 = autotune.TuneCache(p, device_name="B200-test")
    assert c2.get((64, 4096, 2048))["splits"] == 4
    assert autotune.TuneCache(p, device_name="other").get((64, 4096, 2048)) is None
    autotune.activate(c2)
    try:
        assert autotune.lookup(64, 4096, 2048) == (4, 1)
        assert autotune.lookup(1, 2, 3) is None
    finally:
        autotune.activate(None)
    assert autotune.lookup(64, 4096, 2048) is None


def test_candidates_respect_kernel_limits():
    assert autotune.candidates(512, 4096, 4096) == [(1, 0)]          # too many rows to swap
    assert autotune.candidates(64, 1000, 4096) == [(1, 0)]           # N not a multiple of 128
    c = autotune.candidates(64, 4096, 256)                            # 4 K-blocks: splits <= 2
    assert (2, 1) in c and (4, 1) not in c


def test_model_shapes():
    from mod_b200.config import get_preset

    cfg = get_preset("tiny-dense")
    sh = autotune.model_linear_shapes(cfg, [1, 64])
    H = cfg.hidden_size
    assert (64, cfg.q_size + 2 * cfg.kv_size, H) in sh and (1, H, cfg.intermediate_size) in sh


@pytest.mark.gpu
def test_tuned_linear_matches_reference(tmp_path):
    from mod_b200.ops import native

    c = autotune.TuneCache(str(tmp_path / "t.json"))
    e = autotune.tune_linear(64, 1024, 2048, c, reps=5)
    assert e["splits"] in autotune.SPLITS and len(e["trials"]) >= 2
    c.save()
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(64, 2048, device="cuda", generator=g).bfloat16()
    w = (torch.randn(1024, 2048, device="cuda", generator=g) * 0.02).bfloat16()
    ref = x.float() @ w.float().t()
    autotune.activate(autotune.TuneCache(c.path))
    try:
        y = native.linear(x, w, workspace=torch.empty(16 * 64 * 1024, device="cuda"))
    finally:
        autotune.activate(None)
    torch.cuda.synchronize()
    tol = 2e-2 * ref.abs().max().item()
    assert (y.float() - ref).abs().max().item() < tol
