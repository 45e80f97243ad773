"""Sampler, memory manager, KV swap, CLI, metrics, runtime config."""
import json
import subprocess
import sys

import pytest
import torch

from mod_b200.config.runtime import ConfigError, RuntimeConfig, load_runtime, validate
from mod_b200.engine.sampler import Sampler, filter_logits
from mod_b200.engine.sequence import SamplingParams, Sequence


def test_filter_top_k_top_p():
    logits = torch.tensor([[3.0, 2.0, 1.0, 0.0]])
    f = filter_logits(logits, torch.tensor([1.0]), torch.tensor([2]), torch.tensor([1.0]))
    assert torch.isinf(f[0, 2:]).all() and not torch.isinf(f[0, :2]).any()
    p = torch.softmax(logits, -1)[0]
    f = filter_logits(logits, torch.tensor([1.0]), torch.tensor([0]), torch.tensor([float(p[0]) + 1e-3]))
    assert not torch.isinf(f[0, :2]).any() and torch.isinf(f[0, 2:]).all()


def test_sampler_seeded_and_greedy_mix():
    s = Sampler()
    logits = torch.randn(3, 50)
    seqs = [Sequence(prompt=[1], params=SamplingParams(temperature=0.0)),
            Sequence(prompt=[1], params=SamplingParams(temperature=1.0, seed=7)),
            Sequence(prompt=[1], params=SamplingParams(temperature=0.7, top_k=5, seed=3))]
    a = s(logits, seqs)
    assert a[0] == logits[0].argmax()
    assert a[2] in logits[2].topk(5).indices
    s2 = Sampler()
    assert torch.equal(s2(logits, seqs), a)    # same seeds -> same draws


def test_runtime_config_layers(tmp_path, monkeypatch):
    p = tmp_path / "rt.yaml"
    p.write_text("runtime: {max_batch: 7, comm: nccl}\n")
    monkeypatch.setenv("MB_MAX_MODEL_LEN", "999")
    cfg = load_runtime(str(p), profile="balanced", overrides={"tp": 2})
    assert (cfg.max_batch, cfg.comm, cfg.max_model_len, cfg.tp, cfg.kv_mem_fraction) == (7, "nccl", 999, 2, 0.8)
    monkeypatch.setenv("PIO_MAX_BATCH", "5")          # the reference-style prefix is read too...
    monkeypatch.setenv("PIO_SEED", "3")
    monkeypatch.setenv("MB_SEED", "4")                # ...and MB_* wins where both are set
    cfg = load_runtime(overrides={"tp": 1})
    assert (cfg.max_batch, cfg.seed) == (5, 4)
    with pytest.raises(ConfigError):
        validate(RuntimeConfig(backend="nope"))
    with pytest.raises(ConfigError):
        validate(RuntimeConfig(backend="cpu", device="cuda"))


def test_cli_list_and_info():
    r = subprocess.run([sys.executable, "-m", "mod_b200", "info", "qwen3-30b-a3b"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    info = json.loads(r.stdout)
    assert 29e9 < info["parameters"] < 32e9 and 2.5e9 < info["active_parameters"] < 3.7e9
    r = subprocess.run([sys.executable, "-m", "mod_b200", "list"], capture_output=True, text=True)
    assert "Qwen3-VL-2B" in r.stdout


def test_memory_manager_and_kv_swap_cpu():
    from mod_b200.config import get_preset
    from mod_b200.engine.kv_cache import KVCache
    from mod_b200.runtime.memory import KVSwapper, OutOfBudget, UnifiedMemoryManager

    m = UnifiedMemoryManager("cpu")
    n = m.plan_kv_blocks(bytes_per_block=1 << 20, weights_bytes=1 << 20, workspace_bytes=1 << 20)
    assert n > 0
    m.charge("weights", 1 << 20)
    with pytest.raises(OutOfBudget):
        m.charge("weights", 1)
    cfg = get_preset("tiny-dense")
    kv = KVCache(cfg, 8, "cpu", dtype=torch.float32)
    for t in kv.k + kv.v:
        t.normal_()
    before = [t[[2, 5]].clone() for t in kv.k + kv.v]
    sw = KVSwapper(kv)
    sw.swap_out(1, [2, 5])
    for t in kv.k + kv.v:
        t.zero_()
    sw.swap_in(1, [6, 7])
    after = [t[[6, 7]] for t in kv.k + kv.v]
    assert all(torch.equal(a, b) for a, b in zip(after, before))


def test_serving_metrics_fields():
    from mod_b200.utils.metrics import ServingMetrics

    m = ServingMetrics()
    s = Sequence(prompt=[1], output=[1, 2, 3])
    s.t_arrival, s.t_first_token, s.t_finish = 0.0, 0.1, 0.3
    m.record_sequence(s)
    d = m.summary(wall_s=1.0)
    for k in ("avg_inference_time", "std", "avg_memory_usage", "peak_memory_usage", "tokens_per_second", "num_runs",
              "successful_runs"):
        assert k in d
    assert d["tokens_per_second"] == 3.0 and abs(d["tpot_p50_s"] - 0.1) < 1e-9
