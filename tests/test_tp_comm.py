"""Host-side parts of the tensor-parallel boundary flavours (no GPU needed)."""
import pytest
import torch

from mod_b200.parallel.tp import exchange_layout, make_tp_comm, padded_tokens


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("hidden,max_tokens", [(4096, 64), (2048, 128), (4096, 16384), (1024, 7)])
def test_exchange_layout_regions_aligned_and_disjoint(world, hidden, max_tokens):
    L = exchange_layout(hidden, max_tokens, world)
    N, cap, H = world, L["cap"], hidden
    assert cap * world == padded_tokens(max_tokens, world) >= max_tokens
    regions = [("ag_off", N * cap * H * 2), ("rs_off", N * cap * H * 2), ("ag_flag_off", N * 4),
               ("rs_flag_off", N * 4), ("am_off", N * L["am_cap"] * 8), ("am_flag_off", N * 4)]
    end = 0
    for name, size in regions:
        # multimem vector ops and 16-byte stores need 16-byte aligned rows; regions start on 256 bytes
        assert L[name] % 256 == 0 and L[name] >= end, (name, L)
        end = L[name] + size
    assert L["total"] >= end and L["total"] % 256 == 0
    assert (H * 2) % 16 == 0


def test_make_tp_comm_rejects_unknown_flavour():
    with pytest.raises(ValueError, match="unknown tensor-parallel boundary flavour"):
        make_tp_comm("ring", 1024, 16)


def test_nvls_not_supported_without_a_process_group_or_gpu():
    from mod_b200.parallel.symm import nvls_supported

    assert nvls_supported() is False  # no CUDA device / no process group here: the P2P flavour is chosen


def test_nccl_flavour_is_the_baseline_class():
    from mod_b200.parallel.tp import NcclTP

    assert isinstance(make_tp_comm("nccl", 1024, 16), NcclTP)
