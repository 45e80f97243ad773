"""Allocation-free decode-attention entry point (C ABI) vs the torch entry point.

`mb_attn_decode_noalloc` serves callers that cannot allocate GPU memory
(someone else's graph capture in progress, caller-owned-buffer runtimes, C
callers without torch).  It keeps its split-KV scratch in a fixed device array
instead of a caller workspace.  Its results are checked against a plain fp32
torch paged-attention computation.  This file is collected last so a failure here
does not hide any other test's result.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import mod_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.mb_attn_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_void_p]
    lib.mb_noalloc_last_error.restype = ctypes.c_char_p
    lib.mb_attn_decode_noalloc_max_scratch_floats.restype = ctypes.c_size_t
    return lib


def _call(lib, q, kc, vc, bt, ctx, out, splits, scale):
    B, Hq, D = q.shape
    return lib.mb_attn_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), ctx.data_ptr(),
                                      out.data_ptr(), B, Hq, kc.shape[1], D, bt.shape[1], splits, scale,
                                      torch.cuda.current_stream().cuda_stream)


def _fp32_reference(q, kc, vc, bt, ctx, scale):
    """Plain fp32 paged decode attention: gather each sequence's K/V rows from
    its block table (K blocks [Hkv, 16, D], V blocks [Hkv, D, 16]) and softmax."""
    B, Hq, D = q.shape
    Hkv = kc.shape[1]
    G = Hq // Hkv
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        n = min(int(ctx[b]), 16 * bt.shape[1])
        nb = -(-n // 16)
        blocks = bt[b, :nb].long()
        k = kc[blocks].float().permute(0, 2, 1, 3).reshape(nb * 16, Hkv, D)[:n]
        v = vc[blocks].float().permute(0, 3, 1, 2).reshape(nb * 16, Hkv, D)[:n]
        qb = q[b].float().view(Hkv, G, D)
        p = torch.softmax(torch.einsum("hgd,nhd->hgn", qb, k) * scale, dim=-1)
        out[b] = torch.einsum("hgn,nhd->hgd", p, v).reshape(Hq, D)
    return out


@pytest.mark.parametrize("D,Hq,Hkv,splits", [(128, 32, 4, 4), (128, 32, 4, 1), (64, 16, 4, 3), (256, 16, 2, 2)])
def test_noalloc_matches_fp32_reference_twice(cuda, D, Hq, Hkv, splits):
    lib = _lib()
    torch.manual_seed(11)
    B, nb, maxb = 6, 96, 16
    scale = 1.0 / math.sqrt(D)
    for call in range(2):  # two calls in a row: the shared scratch keeps the previous call's contents
        kc = torch.randn(nb, Hkv, 16, D, device=cuda).bfloat16()
        vc = torch.randn(nb, Hkv, D, 16, device=cuda).bfloat16()
        q = torch.randn(B, Hq, D, device=cuda).bfloat16()
        bt = torch.stack([torch.randperm(nb)[:maxb] for _ in range(B)]).int().to(cuda)
        # the last sequence claims more tokens than its 16-entry block-table row addresses:
        # the kernel clamps it to 16 * max_blocks = 256 tokens
        ctx = torch.tensor([1, 40, 255, 17, 100, 300], dtype=torch.int32, device=cuda) - call
        ref = _fp32_reference(q, kc, vc, bt, ctx.cpu(), scale)
        out = torch.full_like(q, float("nan"))
        rc = _call(lib, q, kc, vc, bt, ctx, out, splits, scale)
        torch.cuda.synchronize()
        assert rc == 0, lib.mb_noalloc_last_error()
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


def test_noalloc_matches_torch_entry_point(cuda):
    """Same result as the torch-facing entry point that takes a caller workspace."""
    from mod_b200.ops import native

    lib = _lib()
    torch.manual_seed(5)
    B, Hq, Hkv, D, nb, maxb, splits = 4, 32, 4, 128, 64, 16, 4
    kc = torch.randn(nb, Hkv, 16, D, device=cuda).bfloat16()
    vc = torch.randn(nb, Hkv, D, 16, device=cuda).bfloat16()
    q = torch.randn(B, Hq, D, device=cuda).bfloat16()
    bt = torch.stack([torch.randperm(nb)[:maxb] for _ in range(B)]).int().to(cuda)
    ctx = torch.tensor([3, 77, 200, 256], dtype=torch.int32, device=cuda)
    ws = torch.empty(B * Hq * splits * (D + 1), device=cuda, dtype=torch.float32)
    ref = native.attn_decode(q, kc, vc, bt, ctx, splits=splits, workspace=ws, scale=1.0 / math.sqrt(D))
    out = torch.empty_like(q)
    assert _call(lib, q, kc, vc, bt, ctx, out, splits, 1.0 / math.sqrt(D)) == 0, lib.mb_noalloc_last_error()
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_oversized_request(cuda):
    lib = _lib()
    cap = lib.mb_attn_decode_noalloc_max_scratch_floats()
    B, Hq, Hkv, D = 4, 32, 4, 128
    splits = cap // (B * Hq * (D + 1)) + 1
    q = torch.zeros(B, Hq, D, device=cuda, dtype=torch.bfloat16)
    kc = torch.zeros(2, Hkv, 16, D, device=cuda, dtype=torch.bfloat16)
    bt = torch.zeros(B, 1, device=cuda, dtype=torch.int32)
    ctx = torch.ones(B, device=cuda, dtype=torch.int32)
    out = torch.empty_like(q)
    vc = torch.zeros(2, Hkv, D, 16, device=cuda, dtype=torch.bfloat16)
    rc = _call(lib, q, kc, vc, bt, ctx, out, int(splits), 0.1)
    assert rc == 2
    assert b"maximum" in lib.mb_noalloc_last_error()


def test_noalloc_rejects_unsupported_head_dim(cuda):
    lib = _lib()
    q = torch.zeros(1, 4, 96, device=cuda, dtype=torch.bfloat16)
    kc = torch.zeros(1, 4, 16, 96, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros(1, 4, 96, 16, device=cuda, dtype=torch.bfloat16)
    bt = torch.zeros(1, 1, device=cuda, dtype=torch.int32)
    ctx = torch.ones(1, device=cuda, dtype=torch.int32)
    assert _call(lib, q, kc, vc, bt, ctx, torch.empty_like(q), 1, 0.1) == 3
    assert b"head_dim" in lib.mb_noalloc_last_error()
