"""Preemption with KV swap: a sequence preempted for KV space keeps its KV in
host memory and resumes by copying it back, with no recomputation; its tokens
equal those of an engine that never preempts.  The KV pool size comes from
the engine's unified memory manager."""
import torch

from mod_b200.config import get_preset
from mod_b200.engine import SamplingParams
from mod_b200.engine.llm_engine import LLMEngine
from mod_b200.models.weights import random_weights


def _engine(num_blocks, kv_swap=True):
    cfg = get_preset("tiny-dense")
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=0)
    return LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=4, max_model_len=96,
                     num_blocks=num_blocks, kv_swap=kv_swap)


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, 512, (n,), generator=g).tolist() for n in (30, 17, 25, 9)]


def test_preempted_sequences_resume_from_swapped_kv():
    params = SamplingParams(max_new_tokens=40, ignore_eos=True)
    ref = _engine(64).generate(_prompts(), params)            # room for everyone: no preemption
    eng = _engine(14)                                          # 14 blocks of 16 tokens: decode must preempt
    prefill_tokens = []
    orig = eng.runner.prefill

    def counting_prefill(seqs, qls, *a, **k):
        prefill_tokens.append(sum(qls))
        return orig(seqs, qls, *a, **k)

    eng.runner.prefill = counting_prefill
    out = eng.generate(_prompts(), params)
    st = eng.stats()
    assert st["preempted"] > 0 and st["swapped_out"] == st["preempted"] and st["resumed"] == st["swapped_out"]
    assert out == ref
    # every prompt token was prefilled exactly once: resumed sequences were not recomputed
    assert sum(prefill_tokens) == sum(len(p) for p in _prompts())
    assert not eng.swapper.saved


def test_without_swap_preemption_recomputes():
    params = SamplingParams(max_new_tokens=40, ignore_eos=True)
    ref = _engine(64).generate(_prompts(), params)
    eng = _engine(14, kv_swap=False)
    out = eng.generate(_prompts(), params)
    assert eng.stats()["preempted"] > 0 and eng.stats()["swapped_out"] == 0
    assert out == ref


def test_memory_manager_owns_kv_budget():
    eng = _engine(None)
    rep = eng.memory.report()
    assert rep["kv"]["budget"] > 0 and "host_swap" in rep
