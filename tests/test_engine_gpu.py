"""Native (sm_100a) engine path vs the fp32 oracle and vs the torch baseline."""
import pytest
import torch

from mod_b200.config import get_preset
from mod_b200.engine import SamplingParams
from mod_b200.engine.llm_engine import LLMEngine
from mod_b200.models import oracle
from mod_b200.models.weights import random_weights
from tests.test_engine_cpu import decisive

pytestmark = pytest.mark.gpu


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0).item()


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe", "tiny-glm", "tiny-next"])
def test_native_prefill_and_decode_logits_match_oracle(cuda, name):
    cfg = get_preset(name)
    w = decisive(random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0))
    eng = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=4, max_model_len=128)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (33, 17, 50)]
    ids = [eng.add_request(p[:-1], SamplingParams(max_new_tokens=4)) for p in prompts]
    sched = eng.scheduler.schedule()
    logits_p = eng.runner.prefill(sched.seqs, sched.query_lens, return_logits=True)
    seqs = [eng.seqs[i] for i in ids]
    for s, p in zip(seqs, prompts):
        s.output.append(p[-1])           # force the last prompt token as the next input
    sched = eng.scheduler.schedule()
    assert sched.is_decode
    logits_d = eng.runner.decode(seqs, return_logits=True)
    for b, p in enumerate(prompts):
        ref = oracle.forward(cfg, w, torch.tensor([p], device=cuda))[0]
        assert _cos(logits_p[b], ref[-2]) > 0.995
        assert _cos(logits_d[b], ref[-1]) > 0.995
        assert (logits_d[b] - ref[-1]).abs().max().item() < 0.1


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe"])
def test_native_graph_decode_matches_eager(cuda, name):
    cfg = get_preset(name)
    w = decisive(random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0))
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (12, 30, 7)]
    outs = []
    for graphs in (False, True):
        eng = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=4, max_model_len=128,
                        use_graphs=graphs)
        outs.append(eng.generate(prompts, SamplingParams(max_new_tokens=12)))
    assert outs[0] == outs[1]


@pytest.mark.parametrize("name", ["tiny-next", "tiny-moe"])
def test_int8_engine_matches_torch(cuda, name):
    """int8 weight-only engine (native W8 GEMMs, DeltaNet kernels) vs the torch
    backend on the same quantised weights: identical greedy tokens."""
    from mod_b200.config import get_preset
    from mod_b200.engine import SamplingParams
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.weights import random_weights

    cfg = get_preset(name)
    outs = {}
    for be in ("torch", "native"):
        w = random_weights(cfg, device=cuda, seed=11)
        decisive(w)
        eng = LLMEngine(cfg, weights=w, backend=be, device=cuda, max_batch=4, max_model_len=128, quantization="int8")
        g = torch.Generator().manual_seed(2)
        ps = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 17, 33)]
        ids = [eng.add_request(p, SamplingParams(max_new_tokens=8, ignore_eos=True)) for p in ps]
        while eng.has_unfinished():
            eng.step()
        outs[be] = [eng.seqs[i].output for i in ids]
    agree = sum(a == b for x, y in zip(outs["torch"], outs["native"]) for a, b in zip(x, y))
    total = sum(len(x) for x in outs["torch"])
    assert agree >= 0.9 * total, (outs, agree, total)
