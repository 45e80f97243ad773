"""Cluster split-K decode GEMM (DSMEM reduction) and its fused QKV + RoPE +
QK-norm + KV-write epilogue, against plain fp32 torch references."""
import pytest
import torch

from mod_b200.ops import reference as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,K,N", [(1, 2048, 128), (16, 2048, 5120), (37, 4096, 2048), (128, 2048, 5120),
                                   (64, 768, 2048)])
@pytest.mark.parametrize("cs", [0, 1, 2, 8])
def test_linear_cluster_matches_fp32(cuda, T, K, N, cs):
    from mod_b200.ops import native

    if cs and (K // 64) // cs < 1:
        pytest.skip("fewer K blocks than CTAs")
    torch.manual_seed(T + K + N + cs)
    x = torch.randn(T, K, device=cuda).bfloat16()
    w = (torch.randn(N, K, device=cuda) * 0.02).bfloat16()
    res = torch.randn(T, N, device=cuda).bfloat16()
    for r in (None, res):
        y = native.linear_cluster(x, w, residual=r, cs=cs)
        ref = x.float() @ w.float().t() + (0 if r is None else r.float())
        torch.cuda.synchronize()
        torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * max(1.0, ref.abs().max().item()) / 8)


@pytest.mark.parametrize("T,Hq,Hkv,rot", [(16, 32, 4, 128), (128, 32, 4, 128), (5, 8, 2, 64)])
def test_qkv_rope_cluster_matches_unfused(cuda, T, Hq, Hkv, rot):
    from mod_b200.ops import native

    torch.manual_seed(T + Hq)
    K, D, bs, nblk = 2048, 128, 16, 64
    x = torch.randn(T, K, device=cuda).bfloat16()
    w = (torch.randn((Hq + 2 * Hkv) * D, K, device=cuda) * 0.02).bfloat16()
    qw = (1 + 0.1 * torch.randn(D, device=cuda)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, device=cuda)).bfloat16()
    pos = torch.randint(0, 4000, (T,), device=cuda, dtype=torch.int32)
    invf = R.inv_freq(rot, 1e6, device=cuda)
    slots = torch.randperm(nblk * bs, device=cuda)[:T].int()
    slots[0] = -1  # a padded row: no KV write
    kc0 = torch.randn(nblk, Hkv, bs, D, device=cuda).bfloat16()
    vc0 = torch.randn(nblk, Hkv, D, bs, device=cuda).bfloat16()
    # reference: fp32 GEMM rounded to bf16 (the projection output), then the torch RoPE/QK-norm path
    qkv = (x.float() @ w.float().t()).bfloat16()
    q_ref = torch.empty(T, Hq, D, device=cuda, dtype=torch.bfloat16)
    kc_ref, vc_ref = kc0.clone(), vc0.clone()
    R.rope_qknorm(qkv, qw, kw, pos, invf, slots, q_ref, kc_ref, vc_ref, Hq, Hkv, D, rot, 1e-6)
    q = torch.empty_like(q_ref)
    kc, vc = kc0.clone(), vc0.clone()
    native.qkv_rope_cluster(x, w, qw, kw, pos, invf, slots, q, kc, vc, Hq, Hkv, rot, 1e-6)
    torch.cuda.synchronize()
    torch.testing.assert_close(q.float(), q_ref.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(kc.float(), kc_ref.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(vc.float(), vc_ref.float(), rtol=3e-2, atol=3e-2)
    from mod_b200.ops import check_status

    check_status()


@pytest.mark.parametrize("T,K,N", [(1, 2048, 128), (16, 2048, 5120), (100, 1024, 384), (128, 2048, 2048)])
def test_linear_cluster_w8_matches_fp32(cuda, T, K, N):
    from mod_b200.ops import native
    from mod_b200.ops.quant import quantize_int8

    torch.manual_seed(T + N)
    x = torch.randn(T, K, device=cuda).bfloat16()
    qw = quantize_int8(torch.randn(N, K, device=cuda) * 0.05)
    res = torch.randn(T, N, device=cuda).bfloat16()
    y = native.linear_cluster_w8(x, qw.q, qw.scale, residual=res)
    ref = x.float() @ (qw.q.float() * qw.scale[:, None]).t() + res.float()
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * max(1.0, ref.abs().max().item()) / 8)


def test_linear_cluster_flag_wait(cuda):
    """The tensor-parallel form: x is a gathered buffer and the producer waits on per-rank
    flags.  Flags already at the epoch: same result as without the wait.  A flag that never
    arrives: the bounded wait gives up (about 1 s), records a status code, and the context
    stays usable."""
    import time

    from mod_b200.ops import check_status, native

    check_status()
    torch.manual_seed(5)
    T, K, N, ranks = 16, 2048, 1024, 4
    x = torch.randn(T, K, device=cuda).bfloat16()
    w = (torch.randn(N, K, device=cuda) * 0.02).bfloat16()
    state = torch.zeros(8, dtype=torch.int32, device=cuda)
    state[0] = 3                                            # boundary epoch
    flags = torch.full((ranks,), 3, dtype=torch.int32, device=cuda)
    y = native.linear_cluster(x, w, wait=(flags.data_ptr(), state, ranks))
    ref = native.linear_cluster(x, w)
    torch.cuda.synchronize()
    check_status()
    torch.testing.assert_close(y, ref, rtol=0, atol=0)
    flags[2] = 2                                            # rank 2 never publishes this boundary
    t0 = time.time()
    native.linear_cluster(x, w, wait=(flags.data_ptr(), state, ranks))
    torch.cuda.synchronize()
    assert 0.5 < time.time() - t0 < 30.0
    with pytest.raises(RuntimeError, match="peer flag wait timed out"):
        check_status()
    torch.testing.assert_close(native.linear_cluster(x, w), ref, rtol=0, atol=0)
    check_status()
