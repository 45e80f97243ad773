"""N-gram speculative decoding: drafts come from earlier occurrences, and the
generated tokens equal plain greedy decoding (torch backend on CPU; native
kernels on the GPU)."""
import pytest
import torch

from mod_b200.engine.speculative import NgramSpeculativeDecoder, ngram_propose


def test_ngram_propose():
    assert ngram_propose([1, 2, 3, 9, 1, 2, 3], 3) == [9, 1, 2]
    assert ngram_propose([5, 6, 7], 2) == []
    assert ngram_propose([4, 4, 4, 4], 2) == [4]        # the latest earlier match is followed by one token
    assert ngram_propose([1, 2, 1, 3, 1], 2, ngram_max=2) == [3, 1]


def _repetitive_prompts(vocab):
    g = torch.Generator().manual_seed(5)
    base = torch.randint(1, vocab, (12,), generator=g).tolist()
    return [base * 3, (base[:5] + [7, 8]) * 4, list(range(3, 30))]


def _engine(backend, device, name="tiny-dense", fp32=False):
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.weights import random_weights

    cfg = get_preset(name)
    w = random_weights(cfg, device=device, dtype=torch.float32, seed=0) if fp32 else None
    return LLMEngine(cfg, weights=w, backend=backend, device=device, max_batch=4, max_model_len=160,
                     use_graphs=False)


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe"])
def test_speculative_equals_greedy_cpu(name):
    from mod_b200.engine.sequence import SamplingParams

    prompts = _repetitive_prompts(500)
    # fp32 weights: the one-token and multi-token paths then agree bit for bit on these shapes
    ref = _engine("torch", "cpu", name, fp32=True).generate(prompts, SamplingParams(max_new_tokens=24))
    dec = NgramSpeculativeDecoder(_engine("torch", "cpu", name, fp32=True), k=4)
    got = dec.generate(prompts, max_new_tokens=24)
    assert got == ref
    assert dec.stats.steps > 0 and dec.stats.emitted >= dec.stats.steps


def test_speculative_rejects_recurrent_models():
    with pytest.raises(ValueError):
        NgramSpeculativeDecoder(_engine("torch", "cpu", "tiny-next"))


@pytest.mark.gpu
def test_speculative_equals_greedy_native():
    from mod_b200.engine.sequence import SamplingParams

    prompts = _repetitive_prompts(500)
    ref = _engine("native", "cuda:0").generate(prompts, SamplingParams(max_new_tokens=24))
    dec = NgramSpeculativeDecoder(_engine("native", "cuda:0"), k=4)
    got = dec.generate(prompts, max_new_tokens=24)
    torch.cuda.synchronize()
    # bf16 logits can tie differently between the one-token and multi-token paths; demand near-identity
    same = sum(a == b for a, b in zip(got, ref))
    assert same >= len(ref) - 1, (got, ref)
    assert dec.stats.steps > 0
