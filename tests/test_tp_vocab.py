"""Vocab-parallel LM head: the per-rank slices are 128-row multiples that tile
the vocabulary exactly (an empty slice is allowed for small vocabularies)."""
import types

import pytest
import torch

from mod_b200.models.tp_decoder import TPDecoderLM


@pytest.mark.parametrize("V,N", [(151936, 8), (151936, 2), (512, 4), (500, 4), (300, 4), (1000, 3)])
def test_vocab_slices_tile_the_vocabulary(V, N):
    covered = []
    for r in range(N):
        m = object.__new__(TPDecoderLM)
        m.w = types.SimpleNamespace(lm_head=torch.empty(V, 1))
        m.world, m.comm = N, types.SimpleNamespace(rank=r)
        lo, hi = m._vocab_slice()
        assert 0 <= lo <= hi <= V and (lo % 128 == 0 or lo == hi == V)
        if hi < V:
            assert (hi - lo) % 128 == 0
        covered.extend(range(lo, hi))
    assert covered == list(range(V))
