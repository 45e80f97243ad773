"""Host-side checks of the NVLS all-gather / reduce-scatter expert-parallel
flavour: the buffer layout, and the placement algorithm of
``ep_agrs_place_kernel`` (warp-chunked counting with lane groups of equal
experts, then a warp-major scan) replayed in Python against a stable sort."""
import random

import pytest

from mod_b200.parallel.ep_agrs import agrs_layout, place_reference


def _kernel_placement(ids, counts, rank, El, cap, K, warps=32, lanes=32):
    """Python replay of the kernel's two passes, lane by lane."""
    pstart, acc = [], 0
    for c in counts:
        pstart.append(acc)
        acc += c * K
    P = acc

    def pair_at(p):
        r = max(i for i in range(len(counts)) if pstart[i] <= p and (i + 1 == len(counts) or pstart[i + 1] > p))
        q = p - pstart[r]
        t, k = divmod(q, K)
        g = r * cap + t
        e = int(ids[g][k]) - rank * El
        return g, k, (e if 0 <= e < El else -1)

    ch = (P + warps - 1) // warps
    wbase = [[0] * El for _ in range(warps)]
    for w in range(warps):                                   # pass 1
        lo, hi = w * ch, min(P, w * ch + ch)
        for p0 in range(lo, hi, lanes):
            es = [pair_at(p)[2] if p < hi else -1 for p in range(p0, p0 + lanes)]
            for e in set(es):
                if e >= 0:
                    wbase[w][e] += es.count(e)
    eoff = [0] * (El + 1)
    for e in range(El):                                      # scan, warp-major within an expert
        run = 0
        for w in range(warps):
            c = wbase[w][e]
            wbase[w][e] = run
            run += c
        eoff[e + 1] = run
    for e in range(El):
        eoff[e + 1] += eoff[e]
    slot = {}
    for w in range(warps):                                   # pass 2
        lo, hi = w * ch, min(P, w * ch + ch)
        for p0 in range(lo, hi, lanes):
            info = [pair_at(p) if p < hi else None for p in range(p0, p0 + lanes)]
            es = [i[2] if i else -1 for i in info]
            for lane, i in enumerate(info):
                if i and i[2] >= 0:
                    e = i[2]
                    below = sum(1 for j in range(lane) if es[j] == e)
                    slot[(i[0], i[1])] = eoff[e] + wbase[w][e] + below
            for e in set(es):
                if e >= 0:
                    wbase[w][e] += es.count(e)
    return eoff, slot


@pytest.mark.parametrize("N,El,K,cap,seed", [(2, 8, 4, 16, 0), (8, 16, 8, 16, 1), (4, 64, 10, 8, 2),
                                             (8, 16, 8, 1, 3), (3, 5, 2, 40, 4)])
def test_kernel_placement_matches_stable_sort(N, El, K, cap, seed):
    rng = random.Random(seed)
    E = N * El
    counts = [rng.randint(0, cap) for _ in range(N)]
    ids = [[rng.randrange(E) for _ in range(K)] for _ in range(N * cap)]
    for rank in range(N):
        want_offs, want_slot = place_reference(ids, counts, rank, El, cap)
        offs, slot = _kernel_placement(ids, counts, rank, El, cap, K)
        assert offs == want_offs
        assert slot == want_slot
        assert sorted(slot.values()) == list(range(offs[-1]))  # dense, no collisions
        assert offs[-1] <= N * cap * K                          # the grouped GEMM input's capacity


@pytest.mark.parametrize("N,cap,K,H", [(2, 16, 8, 2048), (8, 16, 8, 2048), (8, 64, 10, 2048), (4, 3, 4, 256)])
def test_agrs_layout_aligned_and_disjoint(N, cap, K, H):
    L = agrs_layout(N, cap, K, H)
    rows = N * cap
    sizes = [("gx", rows * H * 2), ("gid", rows * K * 4), ("gw", rows * K * 4), ("gcnt", N * 4),
             ("part", rows * H * 2), ("ag_flag", N * 4), ("rs_flag", N * 4)]
    end = 0
    for name, size in sizes:
        assert L[name] % 256 == 0 and L[name] >= end, (name, L)
        end = L[name] + size
    assert L["total"] >= end
