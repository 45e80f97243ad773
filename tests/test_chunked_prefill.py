"""Chunked prefill: tokens equal whole-prompt prefill (attention, MoE and the
recurrent DeltaNet state across chunk boundaries), and a decoding request keeps
producing tokens while a long prompt is prefilled."""
import pytest
import torch

from mod_b200.engine.sequence import SamplingParams


def _engine(name, chunk=None, **kw):
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.weights import random_weights

    cfg = get_preset(name)
    w = random_weights(cfg, dtype=torch.float32, seed=0)
    return LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=4, max_model_len=192,
                     use_graphs=False, prefill_chunk=chunk, **kw)


def _prompts():
    g = torch.Generator().manual_seed(9)
    return [torch.randint(1, 500, (n,), generator=g).tolist() for n in (70, 5, 33, 100)]


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe", "tiny-next"])
@pytest.mark.parametrize("chunk", [16, 23])
def test_chunked_equals_whole_prompt(name, chunk):
    p = SamplingParams(max_new_tokens=6)
    ref = _engine(name).generate(_prompts(), p)
    assert _engine(name, chunk).generate(_prompts(), p) == ref


def test_chunked_with_prefix_caching():
    p = SamplingParams(max_new_tokens=6)
    P = _prompts()
    P = P + [P[0][:64] + [7, 7, 7]]
    ref = _engine("tiny-dense").generate(P, p)
    assert _engine("tiny-dense", 16, prefix_caching=True).generate(P, p) == ref


def test_decode_continues_during_long_prefill():
    eng = _engine("tiny-dense", chunk=16)
    a = eng.add_request(_prompts()[1], SamplingParams(max_new_tokens=40))
    eng.step()                                         # a: prefill -> first token
    b = eng.add_request(_prompts()[3], SamplingParams(max_new_tokens=4))   # 100 tokens: 7 chunks
    steps = []
    while eng.seqs[b].t_first_token is None:
        before = len(eng.seqs[a].output)
        eng.step()
        steps.append(len(eng.seqs[a].output) - before)
    # chunks alternate with decode steps, so a gained tokens while b was prefilling
    assert sum(steps) >= 6 and len(eng.seqs[a].output) > 6
