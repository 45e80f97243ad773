"""Allocation-free decode-attention entry point (C ABI) vs the torch entry point.

`mb_attn_decode_noalloc` serves callers that cannot allocate GPU memory
(someone else's graph capture in progress, caller-owned-buffer runtimes, C
callers without torch).  It keeps its split-KV scratch in a fixed device array
instead of a caller workspace.  This file is collected last so a failure here
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


def test_noalloc_matches_torch_entry_point_twice(cuda):
    from mod_b200.ops import native

    lib = _lib()
    torch.manual_seed(11)
    B, Hq, Hkv, D, nb, maxb, splits = 6, 32, 4, 128, 96, 16, 4
    scale = 1.0 / math.sqrt(D)
    for call in range(2):  # two calls in a row: the shared scratch keeps the previous call's contents
        kc = (torch.randn(nb, Hkv, 16, D, device=cuda)).bfloat16()
        vc = (torch.randn(nb, Hkv, D, 16, device=cuda)).bfloat16()
        q = torch.randn(B, Hq, D, device=cuda).bfloat16()
        bt = torch.stack([torch.randperm(nb)[:maxb] for _ in range(B)]).int().to(cuda)
        ctx = torch.tensor([1, 40, 255, 17, 100, 200][:B], dtype=torch.int32, device=cuda) - call
        ctx.clamp_(min=1)
        ws = torch.empty(B * Hq * splits * (D + 1), device=cuda, dtype=torch.float32)
        ref = native.attn_decode(q, kc, vc, bt, ctx, splits=splits, workspace=ws, scale=scale)
        out = torch.full_like(q, float("nan"))
        rc = _call(lib, q, kc, vc, bt, ctx, out, splits, scale)
        torch.cuda.synchronize()
        assert rc == 0, lib.mb_noalloc_last_error()
        scale_t = max(1.0, ref.float().abs().max().item())
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2 * scale_t)


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
