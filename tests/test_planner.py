"""Placement planner: analytic weight bytes match the allocated random-init
model, and the plans for the BASELINE configs are the intended ones."""
import dataclasses

import pytest
import torch

from mod_b200.config import get_preset
from mod_b200.parallel.planner import GIB, plan, weight_bytes


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe", "tiny-next", "tiny-glm"])
def test_weight_bytes_match_allocation(name):
    from mod_b200.models.weights import random_weights

    cfg = get_preset(name)
    w = random_weights(cfg, dtype=torch.bfloat16)
    got = sum(t.numel() * t.element_size() for _, t in w.tensors())
    est = weight_bytes(cfg).total
    assert abs(est - got) / got < 0.01, (est, got)


def test_baseline_configs():
    p = plan(get_preset("qwen3-30b-a3b"), 8)
    assert p.ep == 8 and p.tp == 1 and p.fits and p.kv_tokens_per_gpu > 128 * 768
    assert plan(get_preset("qwen3-30b-a3b"), 1).fits       # ~61 GB of bf16 weights on one GPU
    p8 = plan(get_preset("qwen3-8b"), 8)
    assert p8.tp == 8 and p8.dp == 1 and p8.fits
    assert plan(get_preset("qwen3-8b"), 6).tp in (2, 4)
    nx = plan(get_preset("qwen3-next"), 8)
    assert nx.ep == 8 and nx.fits
    assert plan(get_preset("qwen3-next"), 1).fits           # ~159 GB of bf16 weights fit 180 GB, with little KV room
    one = plan(get_preset("qwen3-next"), 1, hbm_bytes=141 * 10**9)   # a 141 GB part: layers stream from host
    assert not one.fits and one.offload_layers > 0
    q8 = plan(get_preset("qwen3-next"), 1, hbm_bytes=141 * 10**9, int8=True)
    assert q8.fits and q8.weight_bytes_per_gpu < one.weight_bytes_per_gpu


def test_pipeline_when_a_replica_does_not_fit():
    # one KV head caps tensor parallelism at 1, so 4 GPUs are replicas until the weights need stages
    cfg = dataclasses.replace(get_preset("qwen3-8b"), num_hidden_layers=400, num_key_value_heads=1)
    p = plan(cfg, 4, hbm_bytes=80 * GIB)
    assert p.pp > 1 and sum(p.layers_per_stage) == 400
    assert p.weight_bytes_per_gpu <= 80 * GIB or p.offload_layers > 0


def test_cli_plan(capsys):
    import json

    from mod_b200.cli.main import main

    assert main(["plan", "qwen3-30b-a3b", "--gpus", "8"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["ep"] == 8 and out["fits"]


def test_moe_with_tensor_parallel_attention():
    nx = plan(get_preset("qwen3-next"), 8, attn="tp")           # 16 q / 2 KV heads, 16 / 32 DeltaNet heads
    assert nx.tp == 8 and nx.ep == 8 and nx.fits
    assert nx.weight_bytes_per_gpu < plan(get_preset("qwen3-next"), 8).weight_bytes_per_gpu
    assert plan(get_preset("qwen3-30b-a3b"), 8, attn="tp").tp == 8   # 32 q / 4 KV heads: KV replicated x2
