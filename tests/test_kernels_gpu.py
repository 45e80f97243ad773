"""sm_100a kernels vs PyTorch fp32 references of the same op (bf16 tolerances)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _N():
    from mod_b200.ops import check_status, native

    return native, check_status


def _close(a, b, rtol=2e-2, atol=2e-2):
    # bf16 outputs: absolute slack scales with the tensor's magnitude
    scale = max(1.0, b.float().abs().max().item())
    torch.testing.assert_close(a.float(), b.float(), rtol=rtol, atol=atol * scale)


def _rand(*shape, scale=1.0, dev="cuda"):
    return (torch.randn(*shape, device=dev) * scale).to(torch.bfloat16)


# ------------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("T,K,N", [(1, 256, 128), (7, 512, 384), (64, 2048, 5120), (128, 2048, 2048),
                                   (200, 768, 256), (256, 4096, 1024)])
def test_linear_swap_orientation(cuda, T, K, N):
    native, check = _N()
    torch.manual_seed(0)
    x, w = _rand(T, K), _rand(N, K, scale=0.05)
    ref = x.float() @ w.float().t()
    y = native.linear(x, w)
    check()
    _close(y, ref)
    ws = torch.empty(8 * T * N, device=cuda, dtype=torch.float32)
    for splits in (2, 4):
        y2 = native.linear(x, w, workspace=ws, splits=splits)
        check()
        _close(y2, ref)


@pytest.mark.parametrize("T,K,N", [(300, 512, 384), (1024, 1024, 1000), (4096, 2048, 2048), (129, 256, 16)])
def test_linear_normal_orientation(cuda, T, K, N):
    native, check = _N()
    torch.manual_seed(1)
    x, w = _rand(T, K), _rand(N, K, scale=0.05)
    y = native.linear(x, w)
    check()
    _close(y, x.float() @ w.float().t())


def test_linear_residual(cuda):
    native, check = _N()
    x, w, r = _rand(32, 1024), _rand(512, 1024, scale=0.05), _rand(32, 512)
    y = native.linear(x, w, residual=r)
    check()
    _close(y, x.float() @ w.float().t() + r.float())
    ws = torch.empty(8 * 32 * 512, device=cuda, dtype=torch.float32)
    y = native.linear(x, w, residual=r, workspace=ws, splits=4)
    _close(y, x.float() @ w.float().t() + r.float())


@pytest.mark.parametrize("T,K,I", [(1, 256, 128), (64, 4096, 6144), (128, 2048, 768), (200, 1024, 512)])
def test_swiglu_linear_splitk(cuda, T, K, I):
    native, check = _N()
    torch.manual_seed(9)
    x, w = _rand(T, K), _rand(2 * I, K, scale=0.05)
    y = native.swiglu_linear(x, w)
    check()
    gu = x.float() @ w.float().t()
    _close(y, torch.nn.functional.silu(gu[:, :I]) * gu[:, I:])


@pytest.mark.parametrize("E,I,H,T,k,hint_div", [(8, 128, 256, 16, 2, 1), (16, 768, 2048, 128, 8, 1),
                                                (128, 768, 2048, 128, 8, 1), (4, 256, 512, 700, 2, 1),
                                                (128, 768, 2048, 128, 8, 4), (64, 256, 512, 300, 4, 3)])
def test_grouped_swiglu_and_down(cuda, E, I, H, T, k, hint_div):
    """hint_div > 1 passes a row hint below the largest group (as the engine does), so
    groups span several N tiles of the persistent schedule."""
    native, check = _N()
    torch.manual_seed(2)
    counts = torch.randint(0, 2 * T * k // E + 1, (E,))
    counts[0] = 0  # an empty expert
    R = int(counts.sum())
    offs = torch.zeros(E + 1, dtype=torch.int32)
    offs[1:] = counts.cumsum(0)
    xs = _rand(R, H)
    w13 = _rand(E * 2 * I, H, scale=0.05)
    w2 = _rand(E * H, I, scale=0.05)
    hint = max(1, int(counts.max()) // hint_div)
    h = native.grouped_linear(xs, w13, offs.cuda(), E, True, hint)
    y = native.grouped_linear(h, w2, offs.cuda(), E, False, hint)
    check()
    href = torch.empty(R, I)
    yref = torch.empty(R, H)
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        if a == b:
            continue
        gu = xs[a:b].float().cpu() @ w13[e * 2 * I:(e + 1) * 2 * I].float().cpu().t()
        hh = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        href[a:b] = hh
        yref[a:b] = hh.bfloat16().float() @ w2[e * H:(e + 1) * H].float().cpu().t()
    _close(h.cpu(), href)
    _close(y.cpu(), yref)


# ------------------------------------------------------------------------ norms / rope
@pytest.mark.parametrize("H", [256, 1024, 2048, 4096, 1000])
def test_rmsnorm(cuda, H):
    native, check = _N()
    from mod_b200.ops import reference as R

    x, w, r = _rand(37, H), _rand(H), _rand(37, H)
    _close(native.rmsnorm(x, w, 1e-6), R.rmsnorm(x.float(), w.float(), 1e-6))
    r2 = r.clone()
    out = native.rmsnorm(x, w, 1e-6, residual=r2)
    check()
    rr = (r.float() + x.float())
    _close(r2, rr)
    _close(out, R.rmsnorm(rr, w.float(), 1e-6))


@pytest.mark.parametrize("Hq,Hkv,D,rot,qk", [(32, 4, 128, 128, True), (16, 2, 256, 64, True), (4, 2, 128, 128, False)])
def test_rope_qknorm_paged_write(cuda, Hq, Hkv, D, rot, qk):
    native, check = _N()
    from mod_b200.ops import reference as R

    T, nb = 40, 8
    qkv = _rand(T, (Hq + 2 * Hkv) * D)
    qw = _rand(D) if qk else None
    kw = _rand(D) if qk else None
    pos = torch.randint(0, 5000, (T,), device=cuda, dtype=torch.int32)
    slots = torch.randperm(nb * 16, device=cuda)[:T].int()
    slots[3] = -1
    invf = R.inv_freq(rot, 1e6, device=cuda)
    outs = []
    for impl in (native.rope_qknorm, R.rope_qknorm):
        q = torch.empty(T, Hq, D, device=cuda, dtype=torch.bfloat16)
        kc = torch.zeros(nb, Hkv, 16, D, device=cuda, dtype=torch.bfloat16)
        vc = torch.zeros(nb, Hkv, D, 16, device=cuda, dtype=torch.bfloat16)
        impl(qkv, qw, kw, pos, invf, slots, q, kc, vc, Hq, Hkv, D, rot, 1e-6)
        outs.append((q, kc, vc))
    check()
    for a, b in zip(*outs):
        _close(a, b, rtol=2e-2, atol=3e-2)


# ------------------------------------------------------------------------ attention
@pytest.mark.parametrize("B,Hq,Hkv,D,splits", [(4, 32, 4, 128, 1), (3, 32, 4, 128, 4), (5, 16, 2, 256, 2),
                                               (2, 16, 8, 128, 1), (6, 8, 8, 64, 3)])
def test_attn_decode(cuda, B, Hq, Hkv, D, splits):
    native, check = _N()
    from mod_b200.ops import reference as R

    torch.manual_seed(3)
    nb = 64
    kc, vc = _rand(nb, Hkv, 16, D), _rand(nb, Hkv, D, 16)
    lens = torch.tensor([1, 17, 100, 255, 33, 64][:B], dtype=torch.int32)
    maxb = 16
    bt = torch.stack([torch.randperm(nb)[:maxb] for _ in range(B)]).int()
    q = _rand(B, Hq, D)
    ws = torch.empty(B * Hq * splits * (D + 1), device=cuda, dtype=torch.float32)
    o = native.attn_decode(q, kc, vc, bt.cuda(), lens.cuda(), splits=splits, workspace=ws)
    check()
    ref = R.attn_decode(q.float(), kc.float(), vc.float(), bt.cuda(), lens)
    _close(o, ref)


@pytest.mark.parametrize("B,Hq,Hkv,splits,lens", [(4, 32, 4, 1, (1, 17, 100, 255)), (3, 32, 4, 4, (300, 129, 16)),
                                                  (2, 16, 8, 1, (128, 513)), (5, 8, 8, 3, (1, 2, 3, 700, 64)),
                                                  (2, 64, 4, 2, (77, 1000)), (2, 16, 2, 1, (0, 40))])
@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("dynamic", [True, False])
def test_attn_decode_tc(cuda, B, Hq, Hkv, splits, lens, D, dynamic):
    native, check = _N()
    from mod_b200.ops import reference as R

    if D == 256 and Hq // Hkv > 8:
        pytest.skip("head_dim 256 covers groups up to 8")
    torch.manual_seed(5)
    nb = 160
    kc, vc = _rand(nb, Hkv, 16, D), _rand(nb, Hkv, D, 16)
    lens_t = torch.tensor(lens, dtype=torch.int32)
    maxb = 64
    bt = torch.stack([torch.randperm(nb)[:maxb] for _ in range(B)]).int()
    q = _rand(B, Hq, D)
    ws = torch.empty(B * Hq * splits * (D + 1), device=cuda, dtype=torch.float32)
    o = native.attn_decode_tc(q, kc, vc, bt.cuda(), lens_t.cuda(), splits=splits, workspace=ws, dynamic=dynamic)
    check()
    ref = R.attn_decode(q.float(), kc.float(), vc.float(), bt.cuda(), lens_t.clamp(min=1))
    for b in range(B):
        if lens[b] == 0:
            assert torch.all(o[b] == 0)
        else:
            _close(o[b], ref[b])


@pytest.mark.parametrize("D,causal", [(128, True), (256, True), (64, True), (64, False), (256, False)])
@pytest.mark.parametrize("Hq,Hkv,lens", [(32, 4, [(512, 512), (300, 300), (1, 1)]), (16, 8, [(130, 130), (70, 200)]),
                                         (8, 8, [(129, 1000), (256, 256)])])
def test_attn_prefill_tc(cuda, Hq, Hkv, lens, D, causal):
    """(query_len, context_len) per sequence; context > query means a cached prefix.  Head dims
    64 (ViT), 128, 256 (Qwen3-Next gated attention); causal=False is bidirectional attention."""
    native, check = _N()
    from mod_b200.ops import reference as R

    torch.manual_seed(6)
    nb = 256
    kc, vc = _rand(nb, Hkv, 16, D), _rand(nb, Hkv, D, 16)
    B = len(lens)
    maxb = 64
    bt = torch.stack([torch.randperm(nb)[:maxb] for _ in range(B)]).int()
    cu = [0]
    for ql, _ in lens:
        cu.append(cu[-1] + ql)
    T = cu[-1]
    q = _rand(T, Hq, D)
    out = native.attn_prefill_tc(q, kc, vc, bt.cuda(), torch.tensor(cu, dtype=torch.int32, device=cuda),
                                 torch.tensor([c for _, c in lens], dtype=torch.int32, device=cuda),
                                 max(ql for ql, _ in lens), causal=causal)
    check()
    for b, (ql, ctx) in enumerate(lens):
        k = R.gather_kv(kc, bt[b].cuda(), ctx).float()
        v = R.gather_v(vc, bt[b].cuda(), ctx).float()
        qb = q[cu[b]:cu[b + 1]].float()
        mask = torch.arange(ctx, device=cuda)[None, :] <= (ctx - ql + torch.arange(ql, device=cuda))[:, None]
        if not causal:
            mask = torch.ones_like(mask)
        ref = torch.nn.functional.scaled_dot_product_attention(qb.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                               v.transpose(0, 1)[None], attn_mask=mask[None, None],
                                                               enable_gqa=True)[0].transpose(0, 1)
        _close(out[cu[b]:cu[b + 1]], ref)


# ------------------------------------------------------------------------ MoE routing
def test_moe_route_permute_combine(cuda):
    native, check = _N()
    from mod_b200.ops import reference as R

    torch.manual_seed(4)
    T, E, K, H = 50, 128, 8, 256
    logits = _rand(T, E)
    ids = torch.empty(T, K, dtype=torch.int32, device=cuda)
    wts = torch.empty(T, K, dtype=torch.float32, device=cuda)
    counts = torch.empty(E, dtype=torch.int32, device=cuda)
    offs = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    cursor = torch.empty(E, dtype=torch.int32, device=cuda)
    native.moe_route(logits, K, True, ids, wts, counts, offs, cursor)
    check()
    rid, rw = R.moe_route(logits.float(), K, True)
    assert torch.equal(ids.sort(-1).values, rid.sort(-1).values)
    _close(wts.gather(1, ids.argsort(-1).long()), rw.gather(1, rid.argsort(-1).long()), rtol=1e-3, atol=1e-4)
    assert int(offs[-1]) == T * K
    x = _rand(T, H)
    pos = torch.empty(T, K, dtype=torch.int32, device=cuda)
    xs = torch.empty(T * K, H, dtype=torch.bfloat16, device=cuda)
    native.moe_permute(x, ids, offs, cursor, pos, xs)
    assert torch.equal(xs[pos.long().flatten()], x.repeat_interleave(K, 0))
    # rows of each expert segment belong to that expert
    seg = torch.bucketize(pos.long().flatten(), offs[1:].long(), right=True)
    assert torch.equal(seg.int(), ids.flatten())
    y = _rand(T * K, H)
    res = _rand(T, H)
    out = torch.empty_like(x)
    native.moe_combine(y, pos, wts, res, out)
    ref = (y[pos.long()].float() * wts[..., None]).sum(1) + res.float()
    _close(out, ref)


def test_embed_argmax_verify(cuda):
    native, check = _N()
    table = _rand(1000, 256)
    ids = torch.tensor([0, 5, 999, 123], device=cuda)
    assert torch.equal(native.embed(ids, table), table[ids])
    part = native.embed(ids, table[500:], vocab_start=500)
    assert torch.equal(part[2], table[999]) and torch.all(part[0] == 0)
    logits = _rand(7, 151936)
    logits[3, 77] = 100.0
    idx = native.argmax(logits)
    assert torch.equal(idx, logits.float().argmax(-1))
    d = torch.tensor([[1, 2, 3, 4], [1, 2, 3, 4]], device=cuda)
    t = torch.tensor([[1, 2, 9, 4], [1, 2, 3, 4]], device=cuda)
    assert native.verify_tokens(d, t).tolist() == [2, 4]
    check()


# -------------------------------------------------------------------- DeltaNet
def _dn_inputs(T, Hk, Hv, dk, dv, dev):
    C = 2 * Hk * dk + Hv * dv
    mix, z, ba = _rand(T, C), _rand(T, Hv * dv), _rand(T, 2 * Hv)
    conv_w = _rand(C, 4, scale=0.5)
    A_log = torch.rand(Hv, device=dev) * 2 - 1
    dt_bias = torch.randn(Hv, device=dev) * 0.5
    norm_w = (1 + 0.1 * torch.randn(dv, device=dev)).to(torch.bfloat16)
    return mix, z, ba, conv_w, A_log, dt_bias, norm_w


@pytest.mark.parametrize("Hk,Hv,dk", [(2, 4, 64), (4, 8, 128), (2, 2, 128)])
def test_deltanet_prefill_then_decode(cuda, Hk, Hv, dk):
    """Packed multi-sequence prefill (conv + scan kernels) then decode steps (conv + step
    kernels) against the fp32 chunked / recurrent oracle, states compared too."""
    from mod_b200.models.deltanet import ref_decode, ref_prefill

    native, check = _N()
    torch.manual_seed(3)
    dv, eps, S = dk, 1e-6, 6
    C = 2 * Hk * dk + Hv * dv
    lens = [1, 37, 130, 3]
    slots = torch.tensor([4, 0, 2, 5], device=cuda)
    T = sum(lens)
    mix, z, ba, conv_w, A_log, dt_bias, norm_w = _dn_inputs(T, Hk, Hv, dk, dv, cuda)
    conv = torch.randn(S, C, 3, device=cuda) * 0.3
    ssm = torch.randn(S, Hv, dk, dv, device=cuda) * 0.05
    conv_r, ssm_r = conv.clone(), ssm.clone()
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=cuda)
    seq_of = torch.repeat_interleave(torch.arange(len(lens), dtype=torch.int32), torch.tensor(lens)).to(cuda)
    out = native.deltanet_prefill(mix, z, ba, conv_w, conv, ssm, slots, cu, seq_of, A_log, dt_bias, norm_w,
                                  Hk, Hv, dk, dv, eps)
    check()
    refs = []
    for b, L in enumerate(lens):
        s0 = int(cu[b])
        refs.append(ref_prefill(mix[s0:s0 + L], z[s0:s0 + L], ba[s0:s0 + L], conv_w, A_log, dt_bias, norm_w,
                                conv_r, ssm_r, int(slots[b]), Hk, Hv, dk, dv, eps))
    _close(out, torch.cat(refs))
    torch.testing.assert_close(conv, conv_r, rtol=1e-5, atol=1e-5)
    # head dim 128 runs the chunked scan, whose chunk products take bf16 operands: state error
    # ~1e-2 of the state's magnitude (the token-serial scan keeps fp32 throughout)
    stol = 1e-2 * max(1.0, ssm_r.abs().max().item()) if dk == 128 else 1e-3
    torch.testing.assert_close(ssm, ssm_r, rtol=2e-2 if dk == 128 else 1e-3, atol=stol)
    for step in range(3):
        B = len(lens)
        mix, z, ba, *_ = _dn_inputs(B, Hk, Hv, dk, dv, cuda)
        o = native.deltanet_decode(mix, z, ba, conv_w, conv, ssm, slots, A_log, dt_bias, norm_w, Hk, Hv, dk, dv, eps)
        check()
        r = ref_decode(mix, z, ba, conv_w, A_log, dt_bias, norm_w, conv_r, ssm_r, slots, Hk, Hv, dk, dv, eps)
        _close(o, r)
        torch.testing.assert_close(conv, conv_r, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(ssm, ssm_r, rtol=2e-2 if dk == 128 else 1e-3, atol=stol)


@pytest.mark.parametrize("L", [1, 63, 64, 65, 4096])
@pytest.mark.parametrize("chunked", [True, False])
def test_deltanet_prefill_lengths_with_cached_state(cuda, L, chunked):
    """Prefill of one sequence starting from a non-zero cached state, at lengths around the
    64-token chunk, against the fp32 oracle; the chunked tensor-core scan and the token-serial
    scan (MB_DELTANET_CHUNK=0, read once per process, so run in a child) both."""
    import subprocess
    import sys

    code = f"""
import torch, sys
sys.path.insert(0, {repr(str(__import__('os').path.dirname(__import__('os').path.dirname(__file__))))})
from tests.test_kernels_gpu import _dn_inputs
from mod_b200.ops import native, check_status
from mod_b200.models.deltanet import ref_prefill
torch.manual_seed(9)
cuda = torch.device('cuda:0')
Hk, Hv, dk, L = 2, 4, 128, {L}
C = 2 * Hk * dk + Hv * dk
mix, z, ba, conv_w, A_log, dt_bias, norm_w = _dn_inputs(L, Hk, Hv, dk, dk, cuda)
conv = torch.randn(3, C, 3, device=cuda) * 0.3
ssm = torch.randn(3, Hv, dk, dk, device=cuda) * 0.05
conv_r, ssm_r = conv.clone(), ssm.clone()
slots = torch.tensor([1], device=cuda)
cu = torch.tensor([0, L], dtype=torch.int32, device=cuda)
seq_of = torch.zeros(L, dtype=torch.int32, device=cuda)
out = native.deltanet_prefill(mix, z, ba, conv_w, conv, ssm, slots, cu, seq_of, A_log, dt_bias, norm_w,
                              Hk, Hv, dk, dk, 1e-6)
torch.cuda.synchronize(); check_status()
ref = ref_prefill(mix, z, ba, conv_w, A_log, dt_bias, norm_w, conv_r, ssm_r, 1, Hk, Hv, dk, dk, 1e-6)
err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
serr = ((ssm - ssm_r).abs().max() / ssm_r.abs().max()).item()
assert torch.equal(conv, conv_r) or (conv - conv_r).abs().max().item() < 1e-5
assert err < 3e-2 and serr < 3e-2, (err, serr)
print('ok', err, serr)
"""
    env = dict(__import__("os").environ, MB_DELTANET_CHUNK="1" if chunked else "0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


# ------------------------------------------------------------ int8 weight GEMM
@pytest.mark.parametrize("T,K,N", [(1, 256, 128), (16, 2048, 2048), (100, 1024, 384), (256, 4096, 1024),
                                   (1000, 2048, 512), (4096, 1024, 256)])
def test_linear_w8(cuda, T, K, N):
    from mod_b200.ops.quant import quantize_int8

    native, check = _N()
    torch.manual_seed(5)
    x = _rand(T, K)
    qw = quantize_int8(torch.randn(N, K, device=cuda) * 0.05)
    ref = x.float() @ (qw.q.float() * qw.scale[:, None]).t()
    y = native.linear_w8(x, qw.q, qw.scale)
    check()
    _close(y, ref)
    if T <= 256:
        ws = torch.empty(8 * T * N, device=cuda, dtype=torch.float32)
        r = _rand(T, N)
        y2 = native.linear_w8(x, qw.q, qw.scale, residual=r, workspace=ws)
        check()
        _close(y2, ref + r.float())


@pytest.mark.parametrize("T,K,I", [(8, 1024, 256), (200, 2048, 512)])
def test_linear_w8_swiglu(cuda, T, K, I):
    from mod_b200.ops.quant import quantize_int8

    native, check = _N()
    torch.manual_seed(6)
    x = _rand(T, K)
    qw = quantize_int8(torch.randn(2 * I, K, device=cuda) * 0.05)
    gu = x.float() @ (qw.q.float() * qw.scale[:, None]).t()
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    ws = torch.empty(8 * T * 2 * I, device=cuda, dtype=torch.float32)
    for w in (None, ws):
        y = native.linear_w8(x, qw.q, qw.scale, workspace=w, swiglu=True)
        check()
        _close(y, ref)


def test_linear_w8_grouped(cuda):
    """Grouped (MoE) int8 experts: SwiGLU gate/up then down, vs per-expert fp32."""
    from mod_b200.ops.quant import quantize_int8

    native, check = _N()
    torch.manual_seed(7)
    E, H, I = 8, 512, 256
    counts = torch.tensor([0, 5, 17, 1, 0, 40, 3, 9])
    offs = torch.zeros(E + 1, dtype=torch.int32)
    offs[1:] = counts.cumsum(0)
    R_ = int(offs[-1])
    xs = _rand(R_, H)
    w13 = quantize_int8(torch.randn(E * 2 * I, H, device=cuda) * 0.05)
    w2 = quantize_int8(torch.randn(E * H, I, device=cuda) * 0.05)
    d13 = (w13.q.float() * w13.scale[:, None]).view(E, 2 * I, H)
    d2 = (w2.q.float() * w2.scale[:, None]).view(E, H, I)
    offs_d = offs.to(cuda)
    h = native.linear_w8(xs, w13.q, w13.scale, offs=offs_d, groups=E, swiglu=True, max_rows_per_group=40)
    y = native.linear_w8(h, w2.q, w2.scale, offs=offs_d, groups=E, max_rows_per_group=40)
    check()
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        if a == b:
            continue
        gu = xs[a:b].float() @ d13[e].t()
        he = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        _close(h[a:b], he)
        _close(y[a:b], h[a:b].float() @ d2[e].t())


# -------------------------------------------------------------------- sampling
def test_sample_greedy_and_topk1(cuda):
    native, check = _N()
    torch.manual_seed(8)
    B, V = 16, 151936
    logits = _rand(B, V, scale=3.0)
    z = lambda v, dt: torch.full((B,), v, dtype=dt, device=cuda)  # noqa: E731
    seeds = torch.arange(B, device=cuda, dtype=torch.int64)
    steps = torch.zeros(B, device=cuda, dtype=torch.int64)
    ref = logits.float().argmax(-1)
    g = native.sample_tokens(logits, z(0.0, torch.float32), z(0, torch.int32), z(1.0, torch.float32), seeds, steps)
    check()
    assert torch.equal(g, ref)
    k1 = native.sample_tokens(logits, z(0.7, torch.float32), z(1, torch.int32), z(1.0, torch.float32), seeds, steps)
    assert torch.equal(k1, ref)


@pytest.mark.parametrize("temp,k,p", [(1.0, 0, 1.0), (0.8, 5, 1.0), (1.0, 0, 0.7), (1.3, 6, 0.9)])
def test_sample_distribution(cuda, temp, k, p):
    """Many draws of one row: every token lies in the filtered support and the empirical
    frequencies match the truncated softmax."""
    from mod_b200.engine.sampler import filter_logits

    native, check = _N()
    torch.manual_seed(9)
    V, n = 64, 40000
    row = torch.randn(V, device=cuda) * 1.5
    logits = row[None].expand(n, V).contiguous()
    f = lambda v, dt: torch.full((n,), v, dtype=dt, device=cuda)  # noqa: E731
    seeds = torch.arange(n, device=cuda, dtype=torch.int64) + 12345
    steps = torch.full((n,), 3, device=cuda, dtype=torch.int64)
    toks = native.sample_tokens(logits, f(temp, torch.float32), f(k, torch.int32), f(p, torch.float32), seeds, steps)
    check()
    filt = filter_logits(row[None].float(), torch.tensor([temp], device=cuda), torch.tensor([k], device=cuda),
                         torch.tensor([p], device=cuda))[0]
    probs = torch.softmax(filt, -1)
    support = probs > 0
    assert bool(support[toks].all()), "sampled a filtered-out token"
    freq = torch.bincount(toks, minlength=V).float() / n
    assert (freq - probs).abs().max().item() < 0.015
    again = native.sample_tokens(logits, f(temp, torch.float32), f(k, torch.int32), f(p, torch.float32), seeds,
                                 steps)
    assert torch.equal(toks, again), "same (seed, step) must replay"


# ---------------------------------------------------------------- vision front
@pytest.mark.parametrize("h,w", [(448, 448), (300, 520)])
def test_patchify_matches_torch_preprocess(cuda, h, w):
    from mod_b200.config import get_preset
    from mod_b200.models.vl import preprocess

    native, check = _N()
    vc = get_preset("qwen3-vl").vision
    torch.manual_seed(10)
    imgs = torch.rand(2, 3, h, w, device=cuda)
    ref = preprocess(imgs, vc, 448)
    out = native.patchify(imgs, 448, vc.patch_size, vc.spatial_merge_size, vc.image_mean, vc.image_std)
    check()
    torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=2e-2)


def test_bias_gelu(cuda):
    native, check = _N()
    torch.manual_seed(11)
    y, b = _rand(333, 4096, scale=2.0), _rand(4096)
    ref = torch.nn.functional.gelu(y.float() + b.float(), approximate="tanh")
    native.bias_act(y, b, gelu=True)
    check()
    _close(y, ref)
