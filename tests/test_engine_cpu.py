"""Engine (torch backend, fp32 on CPU) vs the fp32 oracle: greedy token match
for every model family, plus scheduler/KV-cache behaviour."""
import pytest
import torch

from mod_b200.config import get_preset
from mod_b200.engine import SamplingParams
from mod_b200.engine.llm_engine import LLMEngine
from mod_b200.models import oracle
from mod_b200.models.weights import random_weights


def decisive(w):
    """Scales MoE router weights so top-k routing has clear margins: random-init
    routers are near-uniform, and a 1e-6 summation-order difference between two
    correct implementations can otherwise swap the k-th and (k+1)-th expert."""
    for L in w.layers:
        if L.moe is not None:
            L.moe.router.mul_(50.0)
    return w


def _prompts(vocab, lens, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe", "tiny-glm", "tiny-next"])
def test_greedy_matches_oracle(name):
    cfg = get_preset(name)
    w = decisive(random_weights(cfg, device="cpu", dtype=torch.float32, seed=0))
    eng = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=4, max_model_len=64)
    prompts = _prompts(cfg.vocab_size, (5, 9, 3))
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=6))
    ref = [oracle.greedy_generate(cfg, w, torch.tensor([p]), 6)[0].tolist() for p in prompts]
    assert outs == ref


def test_preemption_and_requeue():
    cfg = get_preset("tiny-dense")
    w = decisive(random_weights(cfg, device="cpu", dtype=torch.float32, seed=0))
    # 6 blocks of 16 tokens: three 20-token sequences cannot all grow
    eng = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=3, max_model_len=64, num_blocks=6)
    prompts = _prompts(cfg.vocab_size, (20, 20, 20), seed=3)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=14))
    ref = [oracle.greedy_generate(cfg, w, torch.tensor([p]), 14)[0].tolist() for p in prompts]
    assert outs == ref
    assert eng.scheduler.num_preempted > 0
    assert eng.blocks.num_free == 6


def test_oversized_prompt_fails_cleanly():
    cfg = get_preset("tiny-dense")
    w = decisive(random_weights(cfg, device="cpu", dtype=torch.float32, seed=0))
    eng = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=2, max_model_len=64, num_blocks=2)
    with pytest.raises(RuntimeError, match="does not fit"):
        eng.generate([list(range(100))], SamplingParams(max_new_tokens=2))


def test_kv_cache_lengths_after_prefill_and_decode():
    # reference contract: prefill 5 then decode 1 -> cache holds 5 then 6 tokens (tests/test_kv_cache.py:10-82)
    cfg = get_preset("tiny-dense")
    w = decisive(random_weights(cfg, device="cpu", dtype=torch.float32, seed=0))
    eng = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=1, max_model_len=32)
    rid = eng.add_request(list(range(5)), SamplingParams(max_new_tokens=3))
    eng.step()
    assert eng.seqs[rid].num_cached == 5
    eng.step()
    assert eng.seqs[rid].num_cached == 6


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe", "tiny-glm", "tiny-next"])
def test_cpu_cxx_backend_matches_oracle(name):
    pytest.importorskip("mod_b200._cpu")
    cfg = get_preset(name)
    w = decisive(random_weights(cfg, device="cpu", dtype=torch.float32, seed=0))
    eng = LLMEngine(cfg, weights=w, backend="cpu", device="cpu", max_batch=4, max_model_len=64)
    prompts = _prompts(cfg.vocab_size, (5, 9, 3))
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=6))
    ref = [oracle.greedy_generate(cfg, w, torch.tensor([p]), 6)[0].tolist() for p in prompts]
    assert outs == ref
