"""C++/OpenMP CPU backend, op by op, against the torch fp32 oracle at small
shapes (GQA, causal with cached prefixes, QK-norm, partial rotary), plus the
reference's MoE-primitive contract (routing ids/weights, expert mixture)."""
import math

import pytest
import torch
import torch.nn.functional as F

from mod_b200.ops import reference as R

C = pytest.importorskip("mod_b200._cpu")


def _r(*shape, s=1.0, seed=0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * s


def test_linear_rmsnorm_swiglu_gelu_embed_argmax():
    x, w = _r(7, 96, seed=1), _r(40, 96, s=0.1, seed=2)
    y = torch.empty(7, 40)
    C.linear(x, w, y)
    assert torch.allclose(y, x @ w.t(), atol=1e-4)
    res, nw = _r(7, 96, seed=3), _r(96, seed=4)
    out, res2 = torch.empty(7, 96), res.clone()
    C.rmsnorm(x, res2, nw, out, 1e-6)
    h = x + res
    assert torch.allclose(res2, h, atol=1e-6)
    assert torch.allclose(out, h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * nw, atol=1e-5)
    gu, hs = _r(5, 64, seed=5), torch.empty(5, 32)
    C.swiglu(gu, hs)
    assert torch.allclose(hs, F.silu(gu[:, :32]) * gu[:, 32:], atol=1e-5)
    go = torch.empty(5, 64)
    C.gelu_tanh(gu, go)
    assert torch.allclose(go, F.gelu(gu, approximate="tanh"), atol=1e-5)
    table, ids, eo = _r(50, 16, seed=6), torch.tensor([3, 0, 49, 3]), torch.empty(4, 16)
    C.embed(ids, table, eo)
    assert torch.equal(eo, table[ids])
    lg = _r(3, 1000, seed=7)
    assert torch.equal(C.argmax(lg).long(), lg.argmax(-1))


@pytest.mark.parametrize("Hq,Hkv,D,rot", [(8, 2, 32, 32), (4, 4, 64, 16), (16, 2, 16, 16)])
def test_rope_qknorm_gqa_partial_rotary_and_kv_write(Hq, Hkv, D, rot):
    T, bs, nblk = 6, 4, 5
    qkv = _r(T, (Hq + 2 * Hkv) * D, seed=8)
    qw, kw = 1 + _r(D, s=0.1, seed=9), 1 + _r(D, s=0.1, seed=10)
    pos = torch.tensor([0, 1, 2, 7, 8, 20], dtype=torch.int32)
    invf = R.inv_freq(rot, 1e6)
    slots = torch.tensor([0, 1, 2, 9, -1, 17], dtype=torch.int32)   # -1: no cache write
    outs = []
    for fn in (C.rope_qknorm, R.rope_qknorm):
        q = torch.zeros(T, Hq, D)
        kc, vc = torch.zeros(nblk, Hkv, bs, D), torch.zeros(nblk, Hkv, D, bs)
        fn(qkv, qw, kw, pos, invf, slots, q, kc, vc, Hq, Hkv, D, rot, 1e-6)
        outs.append((q, kc, vc))
    for a, b in zip(*outs):
        assert torch.allclose(a, b, atol=1e-5), (a - b).abs().max()


def test_attn_paged_causal_gqa_cached_prefix():
    Hq, Hkv, D, bs = 8, 2, 32, 4
    ctx = [11, 6, 9]                 # tokens in cache after the step
    qlens = [3, 6, 1]                # new tokens (prefix cached before them)
    nblk = 12
    kc, vc = _r(nblk, Hkv, bs, D, seed=11), _r(nblk, Hkv, D, bs, seed=12)
    bt = torch.tensor([[0, 1, 2, 0], [3, 4, 0, 0], [5, 6, 7, 0]], dtype=torch.int32)
    q = _r(sum(qlens), Hq, D, seed=13)
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    C.attn_paged(q, kc, vc, bt, torch.tensor(ctx, dtype=torch.int32), torch.tensor(qlens, dtype=torch.int32), out,
                 scale)
    o = 0
    for b, (n, ql) in enumerate(zip(ctx, qlens)):
        k = R.gather_kv(kc, bt[b], n)
        v = R.gather_v(vc, bt[b], n)
        qb = q[o:o + ql]
        mask = torch.arange(n)[None, :] <= (n - ql + torch.arange(ql))[:, None]
        ref = F.scaled_dot_product_attention(qb.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                             v.transpose(0, 1)[None], attn_mask=mask[None, None], scale=scale,
                                             enable_gqa=True)[0].transpose(0, 1)
        assert torch.allclose(out[o:o + ql], ref, atol=1e-5), b
        o += ql


@pytest.mark.parametrize("renorm", [True, False])
def test_moe_route_and_experts_contract(renorm):
    T, H, E, I, k = 9, 32, 8, 16, 2
    x, router = _r(T, H, seed=14), _r(E, H, s=0.3, seed=15)
    logits = x @ router.t()
    ids, wts = torch.empty(T, k, dtype=torch.int32), torch.empty(T, k)
    C.moe_route(logits, k, renorm, ids, wts)
    rid, rw = R.moe_route(logits, k, renorm)
    assert torch.equal(ids.sort(-1).values, rid.sort(-1).values)         # same experts per token
    assert torch.allclose(wts.sort(-1).values, rw.sort(-1).values, atol=1e-6)
    w13, w2 = _r(E * 2 * I, H, s=0.2, seed=16), _r(E * H, I, s=0.2, seed=17)
    out = torch.zeros(T, H)
    C.moe_experts(x, ids, wts, w13, w2, 0, E, out)
    ref = R.moe_experts(x, ids, wts, w13, w2, E, I)
    assert torch.allclose(out, ref, atol=1e-4)
    # expert-parallel slice: only experts [4, 8) held here; others contribute nothing
    part = torch.zeros(T, H)
    C.moe_experts(x, ids, wts, w13[4 * 2 * I:], w2[4 * H:], 4, 4, part)
    keep = (ids >= 4).float() * wts
    ref_part = R.moe_experts(x, ids.clamp(min=0), keep, w13, w2, E, I)
    assert torch.allclose(part, ref_part, atol=1e-4)


def test_deltanet_recurrence_and_conv1d():
    from mod_b200.models.deltanet import recurrent_step

    B, T, Hv, dk, dv = 2, 5, 3, 8, 6
    q = F.normalize(_r(B, T, Hv, dk, seed=18), dim=-1)
    k = F.normalize(_r(B, T, Hv, dk, seed=19), dim=-1)
    v, g, beta = _r(B, T, Hv, dv, seed=20), -torch.rand(B, T, Hv) * 0.5, torch.rand(B, T, Hv)
    s0 = _r(B, Hv, dk, dv, s=0.1, seed=21)
    state, out = s0.clone(), torch.empty(B, T, Hv, dv)
    C.deltanet_recurrence(q, k, v, g, beta, state, out)
    S = s0.clone()
    for t in range(T):
        o, S = recurrent_step(q[:, t], k[:, t], v[:, t], g[:, t], beta[:, t], S)
        assert torch.allclose(out[:, t], o, atol=1e-5)
    assert torch.allclose(state, S, atol=1e-5)
    Tc, Cc, K = 7, 5, 4
    x, w, st = _r(Tc, Cc, seed=22), _r(Cc, K, seed=23), _r(Cc, K - 1, seed=24)
    st2, y = st.clone(), torch.empty(Tc, Cc)
    C.conv1d_causal(x, w, st2, y)
    full = torch.cat([st.t(), x], 0).t()[None]                            # [1, C, K-1+T]
    ref = F.conv1d(full, w[:, None, :], groups=Cc)[0].t()
    assert torch.allclose(y, ref, atol=1e-5)
    assert torch.allclose(st2, full[0, :, -(K - 1):])


@pytest.mark.parametrize("oh,ow", [(16, 24), (5, 7), (10, 10)])
def test_resize_bilinear_matches_interpolate(oh, ow):
    img = _r(3, 10, 12, seed=25)
    out = torch.empty(3, oh, ow)
    C.resize_bilinear(img, out)
    ref = F.interpolate(img[None], size=(oh, ow), mode="bilinear", align_corners=False)[0]
    assert torch.allclose(out, ref, atol=1e-5)


@pytest.mark.parametrize("M,K,N", [(1, 1024, 300), (1, 40, 7), (6, 1000, 37), (128, 256, 96)])
def test_linear_bf16_weights_equal_fp32_math(M, K, N):
    x, w = _r(M, K, seed=30), (_r(N, K, seed=31) * 0.05).bfloat16()
    y = torch.empty(M, N)
    C.linear(x, w, y)
    assert torch.allclose(y, x @ w.float().t(), atol=1e-5)


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe", "tiny-next", "tiny-glm"])
def test_cpu_engine_bf16_weights_match_widened_copy(name):
    """bf16 weights (widened in registers) give the same tokens as an fp32 copy of the same values."""
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.engine.sequence import SamplingParams
    from mod_b200.models.weights import random_weights

    def widen(obj):
        for k, v in list(vars(obj).items()):
            if isinstance(v, torch.Tensor):
                if v.dtype == torch.bfloat16:
                    setattr(obj, k, v.float())
            elif isinstance(v, list):
                for e in v:
                    if hasattr(e, "__dict__"):
                        widen(e)
            elif hasattr(v, "__dict__"):
                widen(v)

    cfg = get_preset(name)
    wb = random_weights(cfg, dtype=torch.bfloat16, seed=0)
    wf = random_weights(cfg, dtype=torch.bfloat16, seed=0)
    widen(wf)
    prompts = [[1, 2, 3, 4, 5], [7, 8, 9]]
    p = SamplingParams(max_new_tokens=6)
    a = LLMEngine(cfg, weights=wb, backend="cpu", device="cpu", max_batch=2, max_model_len=64).generate(prompts, p)
    b = LLMEngine(cfg, weights=wf, backend="cpu", device="cpu", max_batch=2, max_model_len=64).generate(prompts, p)
    assert a == b


@pytest.mark.parametrize("M,K,N", [(1, 1024, 300), (1, 40, 7), (6, 1000, 37), (128, 256, 96)])
def test_linear_int8_weights(M, K, N):
    x = _r(M, K, seed=32)
    q = torch.randint(-127, 128, (N, K), generator=torch.Generator().manual_seed(33), dtype=torch.int8)
    sc = torch.rand(N, generator=torch.Generator().manual_seed(34)) * 0.01
    y = torch.empty(M, N)
    C.linear_w8(x, q, sc, y)
    ref = x @ (q.float() * sc[:, None]).t()
    assert torch.allclose(y, ref, atol=1e-4, rtol=1e-5)


def test_cpu_engine_int8_matches_dequantized_weights():
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.engine.sequence import SamplingParams
    from mod_b200.models.weights import random_weights
    from mod_b200.ops.quant import Int8Weight, quantize_model

    cfg = get_preset("tiny-dense")
    wq = random_weights(cfg, dtype=torch.float32, seed=0)
    quantize_model(wq)
    wd = random_weights(cfg, dtype=torch.float32, seed=0)
    quantize_model(wd)
    for L in wd.layers:                    # the same int8 values, dequantized to fp32 up front
        for part in (L.attn, L.mlp):
            for k, v in list(vars(part).items()):
                if isinstance(v, Int8Weight):
                    setattr(part, k, v.q.float() * v.scale[:, None])
    prompts = [[1, 2, 3, 4, 5], [7, 8, 9]]
    p = SamplingParams(max_new_tokens=6)
    a = LLMEngine(cfg, weights=wq, backend="cpu", device="cpu", max_batch=2, max_model_len=64).generate(prompts, p)
    b = LLMEngine(cfg, weights=wd, backend="cpu", device="cpu", max_batch=2, max_model_len=64).generate(prompts, p)
    assert a == b


def test_cpu_moe_int8_experts_match_torch_backend():
    """int8 experts: only the routed experts are widened per call; same tokens as the torch path."""
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.engine.sequence import SamplingParams
    from mod_b200.models.weights import random_weights
    from mod_b200.ops.quant import quantize_model

    cfg = get_preset("tiny-moe")
    w = random_weights(cfg, dtype=torch.float32, seed=0)
    quantize_model(w)
    prompts, p = [[1, 2, 3, 4, 5], [7, 8, 9]], SamplingParams(max_new_tokens=5)
    a = LLMEngine(cfg, weights=w, backend="cpu", device="cpu", max_batch=2, max_model_len=64).generate(prompts, p)
    b = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=2, max_model_len=64).generate(prompts, p)
    assert a == b
