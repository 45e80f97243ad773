"""Reference-compatible Tensor API: every method against plain torch, plus the
reference's own behavioural contracts (MoE primitives, shapes, in-place ops)."""
import math

import pytest
import torch
import torch.nn.functional as F

from mod_b200.compat import Tensor


def T(t):
    return Tensor.from_torch(t.float().clone())  # from_torch shares storage, like torch.from_numpy


def _r(*s, seed=0):
    return torch.randn(*s, generator=torch.Generator().manual_seed(seed))


def test_storage_shape_and_device():
    a = Tensor([2, 3], data=[1, 2, 3, 4, 5, 6])
    assert a.shape == (2, 3) and a.ndim == 2 and a.size == 6 and a.dtype == "float32"
    assert a.to("cpu").to_list() == [1, 2, 3, 4, 5, 6]
    a.fill(2.0)
    assert a.to_list() == [2.0] * 6
    with pytest.raises(ValueError):
        Tensor([2], device="opencl:amd:0")
    with pytest.raises(ValueError):
        a.load([1, 2])


def test_linear_algebra_and_activations():
    x, w, b = _r(3, 8, seed=1), _r(5, 8, seed=2), _r(5, seed=3)
    assert torch.allclose(T(x).linear(T(w), T(b)).data, x @ w.t() + b, atol=1e-5)
    assert torch.allclose(T(x).matmul(T(w), transpose_b=True).data, x @ w.t(), atol=1e-5)
    assert torch.allclose(T(x).add(T(x)).data, 2 * x) and torch.allclose(T(x).mul(3).data, 3 * x)
    assert torch.allclose(T(x).mul(T(x)).data, x * x)
    gu = _r(4, 10, seed=4)
    assert torch.allclose(T(gu).fused_swiglu().data, F.silu(gu[:, :5]) * gu[:, 5:])
    assert torch.allclose(T(gu[:, :5]).swiglu(T(gu[:, 5:])).data, F.silu(gu[:, :5]) * gu[:, 5:])
    assert torch.allclose(T(x).softmax().data, torch.softmax(x, -1))
    assert torch.allclose(T(x).silu().data, F.silu(x)) and torch.allclose(T(x).gelu().data, F.gelu(x, approximate="tanh"))
    nw = _r(8, seed=5)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * nw
    assert torch.allclose(T(x).rms_norm(T(nw)).data, ref, atol=1e-6)
    a, r = T(x), T(x)
    out = a.fused_add_rms_norm(r, T(nw), 1e-6)
    h = 2 * x
    assert torch.allclose(a.data, h) and torch.allclose(out.data, h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * nw, atol=1e-5)
    img, cw = _r(1, 3, 9, 9, seed=6), _r(4, 3, 3, 3, seed=7)
    assert torch.allclose(T(img).conv2d(T(cw), stride=2, padding=1).data, F.conv2d(img, cw, stride=2, padding=1), atol=1e-5)
    assert torch.allclose(T(x).dequantize(T(torch.tensor(0.5))).data, x * 0.5)


def test_shapes_selection_and_slices():
    x = _r(2, 3, 4, seed=8)
    assert T(x).permute([2, 0, 1]).shape == (4, 2, 3)
    assert T(x).reshape([6, 4]).shape == (6, 4)
    with pytest.raises(ValueError):
        T(x).reshape([5, 5])
    v, i = T(x).topk(2)
    rv, ri = torch.topk(x, 2)
    assert torch.equal(v.data, rv) and torch.equal(i.data, ri.float())
    assert torch.equal(T(x).argmax().data, x.argmax(-1).float())
    table = _r(10, 4, seed=9)
    ids = T(torch.tensor([[1, 9], [0, 3]]))
    assert torch.equal(T(table).embed(ids).data, table[torch.tensor([[1, 9], [0, 3]])])
    with pytest.raises(IndexError):
        T(table).embed(T(torch.tensor([10])))
    s = T(x).slice([0, 1, 1], [2, 2, 3])
    assert torch.equal(s.data, x[:, 1:3, 1:4])
    s2 = T(x).slice(T(torch.tensor([1, 0, 0])), [1, 3, 4])
    assert torch.equal(s2.data, x[1:2])
    dst = T(torch.zeros(2, 3, 4))
    dst.set_slice(s, [0, 1, 1])
    assert torch.equal(dst.data[:, 1:3, 1:4], s.data)
    g = T(table).gather(T(torch.tensor([3, 3, 0])))
    assert torch.equal(g.data, table[[3, 3, 0]])
    acc = T(torch.zeros(4, 4))
    acc.scatter_add(T(torch.tensor([1, 1, 3])), T(torch.ones(3, 4)))
    assert acc.data[1].tolist() == [2.0] * 4 and acc.data[3].tolist() == [1.0] * 4


def test_rope_every_head_uses_position_table():
    S, Hq, Hkv, D = 5, 4, 2, 8
    q, k = _r(1, S, Hq, D, seed=10), _r(1, S, Hkv, D, seed=11)
    ang = torch.arange(S)[:, None] * (1e4 ** (-torch.arange(D // 2) / (D // 2)))[None]
    cos, sin = ang.cos(), ang.sin()
    oq, ok = T(q).rope(T(k), T(cos), T(sin))

    def rot(x):
        x1, x2 = x[..., :D // 2], x[..., D // 2:]
        c, s = cos[:, None], sin[:, None]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1)

    assert torch.allclose(oq.data, rot(q), atol=1e-6) and torch.allclose(ok.data, rot(k), atol=1e-6)
    packed = torch.cat([q.reshape(1, S, -1), q.reshape(1, S, -1), q.reshape(1, S, -1)], -1)
    a, b, c = T(packed).fused_split_rope(T(cos), T(sin), Hq, D)
    assert torch.allclose(a.data, rot(q), atol=1e-6) and torch.allclose(c.data, q)


def test_moe_primitives_contract():
    # the reference's MoE dispatch test (sorted by index to hide its OpenMP order): count, gather, scatter back
    x = _r(6, 4, seed=12)
    ids = T(torch.tensor([2.0, 0.0, 2.0, 1.0, 2.0, 0.0]))
    assert ids.count_value(2.0) == 3 and ids.count_value(5.0) == 0
    rows, where = T(x).gather_by_value(ids, 2.0)
    assert where.to_list() == [0.0, 2.0, 4.0] and torch.equal(rows.data, x[[0, 2, 4]])
    assert T(x).gather_by_value(ids, 7.0) == (None, None)
    out = T(torch.zeros(6, 4))
    out.scatter_add_by_index(rows.mul(2.0), where)
    out.scatter_add_by_index(rows, T(torch.tensor([0.0, 99.0, -1.0])))    # out-of-range rows are skipped
    exp = torch.zeros(6, 4)
    exp[[0, 2, 4]] = 2 * x[[0, 2, 4]]
    exp[0] += x[0]
    assert torch.allclose(out.data, exp)


def test_deltanet_recurrence_and_resize():
    B, S, H, D = 1, 4, 2, 3
    q, k, v = _r(B, S, H, D, seed=13), _r(B, S, H, D, seed=14), _r(B, S, H, D, seed=15)
    beta = torch.rand(B, S, H, generator=torch.Generator().manual_seed(16))
    st = T(torch.zeros(B, H, D, D))
    o = T(q).deltanet_recurrence(T(k), T(v), T(beta), st)
    Sm = torch.zeros(B, H, D, D)
    for t in range(S):
        Sm = beta[:, t, :, None, None] * Sm + k[:, t, :, :, None] * v[:, t, :, None, :]
        assert torch.allclose(o.data[:, t], torch.einsum("bhd,bhde->bhe", q[:, t], Sm), atol=1e-5)
    assert torch.allclose(st.data, Sm, atol=1e-5)
    img = _r(3, 8, 10, seed=17)
    r = T(img).resize_image(5, 7)
    assert r.shape == (3, 5, 7)
    assert torch.allclose(r.data, F.interpolate(img[None], size=(5, 7), mode="bilinear", align_corners=False)[0],
                          atol=1e-5)
