"""Prefix caching: requests sharing a prompt prefix reuse its KV blocks, the
tokens equal a run without caching, and a small pool evicts cached blocks."""
import torch

from mod_b200.engine.block_manager import PrefixCachingBlockManager
from mod_b200.engine.sequence import SamplingParams, Sequence


def _engine(caching, num_blocks=None, name="tiny-dense"):
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.weights import random_weights

    cfg = get_preset(name)
    w = random_weights(cfg, dtype=torch.float32, seed=0)
    return LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=4, max_model_len=160,
                     num_blocks=num_blocks, use_graphs=False, prefix_caching=caching)


def _prompts():
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(1, 500, (40,), generator=g).tolist()
    return [shared + torch.randint(1, 500, (n,), generator=g).tolist() for n in (9, 17, 3, 30)]


def test_shared_prefix_reuses_blocks_and_matches():
    P = _prompts()
    p = SamplingParams(max_new_tokens=8)
    ref = [_engine(False).generate([q], p)[0] for q in P]
    eng = _engine(True)
    got = [eng.generate([P[0]], p)[0]]                  # fills the cache
    got += eng.generate(P[1:3], p)                       # two requests adopt the 2 shared blocks
    got += eng.generate([P[3]], p)
    assert got == ref
    assert eng.blocks.hits >= 2 * 3                       # 2 shared full blocks x 3 later requests
    assert eng.blocks.num_free == eng.blocks.num_blocks  # everything released (cached blocks are reusable)


def test_small_pool_evicts_and_preempts_correctly():
    P = _prompts() * 2
    p = SamplingParams(max_new_tokens=12)
    ref = _engine(False, num_blocks=12).generate(P, p)
    eng = _engine(True, num_blocks=12)
    assert eng.generate(P, p) == ref
    assert eng.scheduler.num_preempted > 0 and eng.blocks.hits > 0   # the pool is small enough to preempt


def test_manager_refcounts_and_lru():
    m = PrefixCachingBlockManager(num_blocks=6, block_size=4, max_seqs=4)
    a = Sequence(prompt=list(range(10)))
    assert m.allocate(a, a.length + 1) and a.num_cached == 0 and len(a.blocks) == 3
    a.num_cached = a.length
    m.register(a)                                          # blocks 0-1 full -> cached
    b = Sequence(prompt=list(range(9)) + [99])
    assert m.allocate(b, b.length + 1)
    assert b.blocks[:2] == a.blocks[:2] and b.num_cached == 8 and m.ref[a.blocks[0]] == 2
    m.release(a)
    assert m.ref[b.blocks[0]] == 1 and m.num_free == 6 - 3 - 0  # a's private tail block went back to free
    m.release(b)
    assert len(m.lru) == 2 and m.num_free == 6
    c = Sequence(prompt=[7] * 23)                          # needs all 6 blocks: both cached ones are evicted
    assert m.allocate(c, c.length + 1) and len(c.blocks) == 6 and not m.cache
