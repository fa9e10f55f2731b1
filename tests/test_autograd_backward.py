"""Autograd gradient functions (autograd/ops.rs GradFn::backward).

CPU: the oracle against the reference's own autograd unit tests
(autograd/tests.rs:63-226, :606-652) and against independent numpy
restatements; the C ABI's validation.  GPU: every backward entry point
against the oracle, bit for bit, including NULL gradient outputs, in-place
outputs, unaligned views, host-memory tensors and each branch of
reduce_to_shape.
"""
import ctypes
import math

import numpy as np
import pytest

from rusttorch_b200 import _native as N
from tests import _oracle as O
from tests.test_parity_gpu import assert_bits_equal, edge_values

F = np.float32


def bits(x):
    return np.asarray(x, dtype=F).view(np.uint32)


def ones(n):
    return np.ones(n, F)


# ---- CPU: the reference's autograd tests, through the oracle ----------------
def test_oracle_reference_autograd_kats():
    # test_relu_backward (:158-168): loss = sum(relu(x)) so grad_output = ones
    x = np.array([-2.0, -1.0, 0.0, 1.0, 2.0], F)
    assert O.grad_unary("relu", ones(5), x).tolist() == [0.0, 0.0, 0.0, 1.0, 1.0]
    # test_sigmoid_backward (:171-179): sigmoid(0) = 0.5 -> 0.25
    assert O.grad_unary("sigmoid", ones(1), np.array([0.5], F))[0] == F(0.25)
    # test_tanh_backward (:182-190): tanh(0) = 0 -> 1
    assert O.grad_unary("tanh", ones(1), np.zeros(1, F))[0] == F(1.0)
    # test_add/sub/mul/div_backward (:63-121)
    ga, gb = O.grad_binary("add", ones(3))
    assert ga.tolist() == [1.0] * 3 and gb.tolist() == [1.0] * 3
    ga, gb = O.grad_binary("sub", ones(2))
    assert ga.tolist() == [1.0, 1.0] and gb.tolist() == [-1.0, -1.0]
    ga, gb = O.grad_binary("mul", ones(2), np.array([2, 3], F), np.array([4, 5], F))
    assert ga.tolist() == [4.0, 5.0] and gb.tolist() == [2.0, 3.0]
    ga, gb = O.grad_binary("div", ones(2), np.array([6, 8], F), np.array([2, 4], F))
    assert np.allclose(ga, [0.5, 0.25], atol=1e-5) and np.allclose(gb, [-1.5, -0.5], atol=1e-5)
    # test_sum_backward / test_mean_backward (:193-212)
    assert O.fill_backward(1.0, (4,), False).tolist() == [1.0] * 4
    assert np.allclose(O.fill_backward(1.0, (4,), True), 0.25, atol=1e-5)
    # test_gelu_backward (:606-619): GELU'(0) ~ 0.5, all finite
    g = O.grad_unary("gelu", ones(4), np.array([0.0, 1.0, -1.0, 2.0], F))
    assert abs(g[0] - 0.5) < 0.01 and np.isfinite(g).all()


def test_oracle_gelu_matches_numerical_gradient():
    # test_gelu_numerical_gradient (:622-652), on autograd's own gelu forward
    xs = np.array([0.5, -0.5, 1.5, -1.5], F)
    analytical = O.grad_unary("gelu", ones(4), xs)
    eps = F(1e-4)
    for i in range(4):
        xp, xm = xs.copy(), xs.copy()
        xp[i] += eps
        xm[i] -= eps
        lp = F(0)
        for v in O.autograd_gelu(xp):
            lp = F(lp + v)
        lm = F(0)
        for v in O.autograd_gelu(xm):
            lm = F(lm + v)
        numerical = F(F(lp - lm) / F(F(2.0) * eps))
        assert abs(float(analytical[i]) - float(numerical)) < 1e-3


def _np_gelu_backward(g, x):
    """numpy float32 restatement of ops.rs:3108-3118 with tanh from Python's
    math module rounded once to f32 (glibc tanhf is within 1 ulp of it)."""
    k = F(math.sqrt(float(F(2.0) / F(math.pi))))
    c3 = F(F(3.0) * F(0.044715))
    out = np.empty_like(x)
    for i, xi in enumerate(x):
        inner = F(k * F(xi + F(F(0.044715) * F(F(xi * xi) * xi))))
        t = F(math.tanh(float(inner)))
        sech2 = F(F(1.0) - F(t * t))
        d_inner = F(k * F(F(1.0) + F(F(c3 * xi) * xi)))
        a = F(F(0.5) * F(F(1.0) + t))
        b = F(F(F(F(0.5) * xi) * sech2) * d_inner)
        out[i] = F(g[i] * F(a + b))
    return out


def test_oracle_backward_matches_numpy_restatement():
    n = 4099
    g = O.normal(n, 11, 0, 2.0)
    x = np.concatenate([edge_values(), O.normal(n - edge_values().size, 12, 0, 3.0)])
    y = O.uniform(n, 13, -1.0, 1.0)
    with np.errstate(all="ignore"):
        want = {
            "relu": (g * np.where(x > 0, F(1), F(0))).astype(F),
            "sigmoid": (g * (y * (F(1) - y)).astype(F)).astype(F),
            "tanh": (g * (F(1) - (y * y).astype(F)).astype(F)).astype(F),
        }
        for name, w in want.items():
            saved = x if name == "relu" else y
            assert_bits_equal(O.grad_unary(name, g, saved), w, name)
        a, b = O.normal(n, 14), O.normal(n, 15)
        ga, gb = O.grad_binary("mul", g, a, b)
        assert_bits_equal(ga, (g * b).astype(F), "mul a")
        assert_bits_equal(gb, (g * a).astype(F), "mul b")
        ga, gb = O.grad_binary("div", g, a, b)
        assert_bits_equal(ga, (g / b).astype(F), "div a")
        assert_bits_equal(gb, (g * ((-a) / (b * b).astype(F)).astype(F)).astype(F), "div b")
    xs = O.normal(300, 16, 0, 2.0)
    gs = O.normal(300, 17)
    got = O.grad_unary("gelu", gs, xs)
    want = _np_gelu_backward(gs, xs)
    # one ulp in tanh can move the result by a few ulp where a + b cancels
    assert np.allclose(got, want, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("gshape,oshape", [
    ((5, 7), (1, 7)), ((5, 7), (5, 1)), ((5, 7), (7,)), ((5, 7), (35,)), ((2, 3, 4), (4,)),
    ((2, 3, 4), (2, 1, 4)), ((6,), (1,)), ((3, 4), (3, 4)), ((7,), (3,)), ((2, 2), (5,)),
    ((9, 1), (1, 1)),
])
def test_oracle_reduce_to_shape_matches_python(gshape, oshape):
    grad = O.normal(int(np.prod(gshape)), 21).reshape(gshape)
    rc, got = O.reduce_to_shape(grad, oshape)
    assert rc == 0
    flat = grad.ravel()
    m = int(np.prod(oshape))
    if gshape == oshape or (len(gshape) != 2 or len(oshape) != 2) and flat.size == m:
        want = flat.copy()
    elif len(gshape) == 2 and len(oshape) == 2 and oshape == (1, gshape[1]):
        want = np.zeros(gshape[1], F)
        for r in range(gshape[0]):
            want = (want + grad[r]).astype(F)
    elif len(gshape) == 2 and len(oshape) == 2 and oshape == (gshape[0], 1):
        want = np.zeros(gshape[0], F)
        for r in range(gshape[0]):
            for c in range(gshape[1]):
                want[r] = F(want[r] + grad[r, c])
    else:
        want = np.zeros(m, F)
        for i, v in enumerate(flat):
            want[i % m] = F(want[i % m] + v)
    assert_bits_equal(got.ravel(), want, f"{gshape}->{oshape}")


# ---- CPU: C ABI validation (no device work) -------------------------------
def _desc(shape, dtype=N.F32, device=0):
    return N.Desc(0x1000, shape, dtype, device)


def _err(res):
    assert not res.success
    msg = ctypes.string_at(res.error_msg).decode()
    N.lib().rtc_free_error_message(res.error_msg)
    return res.code, msg


def test_abi_backward_validation_follows_the_reference_ops():
    L = N.lib()
    g, x, bad = _desc([2, 3]), _desc([2, 3]), _desc([3, 2])
    code, msg = _err(L.rtc_relu_backward(g.ref, bad.ref, x.ref))
    assert code == N.SHAPE_MISMATCH and "element-wise multiplication" in msg
    # mul: grad_a checks (g, b) first; with grad_a NULL only (g, a) is checked
    code, msg = _err(L.rtc_mul_backward(g.ref, x.ref, bad.ref, x.ref, None))
    assert code == N.SHAPE_MISMATCH
    code, msg = _err(L.rtc_mul_backward(g.ref, bad.ref, x.ref, None, x.ref))
    assert code == N.SHAPE_MISMATCH
    # div: grad_b's (-a)/(b*b) needs a and b of one shape
    code, msg = _err(L.rtc_div_backward(g.ref, x.ref, bad.ref, None, x.ref))
    assert code == N.SHAPE_MISMATCH and "element-wise division" in msg
    d64 = _desc([2, 3], N.F64)
    code, msg = _err(L.rtc_div_backward(g.ref, x.ref, d64.ref, x.ref, None))
    assert code == N.DTYPE_MISMATCH
    # item() on a grad_output of several elements
    code, msg = _err(L.rtc_sum_backward(g.ref, x.ref))
    assert code == N.INVALID_ARGUMENT and msg.endswith(
        "item() requires a single-element tensor, got 6 elements")
    host = _desc([2, 3], device=-1)
    code, msg = _err(L.rtc_broadcast_add_backward(host.ref, x.ref, None))
    assert code == N.INVALID_ARGUMENT and "device" in msg
    # no gradient wanted: nothing to do, no device needed
    assert L.rtc_mul_backward(g.ref, x.ref, x.ref, None, None).success
    assert L.rtc_sub_backward(g.ref, None, None).success


# ---- GPU --------------------------------------------------------------------
SIZES = [1, 7, 1000, (1 << 20) + 3]


def _inputs(n, seed):
    g = O.normal(n, seed, 0, 2.0)
    x = O.normal(n, seed + 1, 0, 3.0)
    e = edge_values()
    k = min(n, e.size)
    x[:k] = e[:k]
    return g, x


@pytest.mark.gpu
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("name", ["relu", "sigmoid", "tanh", "gelu"])
def test_gpu_grad_unary(name, n):
    import rusttorch_b200 as rt
    g, x = _inputs(n, 30)
    saved = x
    if name == "sigmoid":
        saved = O.unary("sigmoid", x)
    elif name == "tanh":
        saved = O.unary("tanh", x)
    want = O.grad_unary(name, g, saved)
    got = getattr(rt, name + "_backward")(rt.Tensor.from_numpy(g), rt.Tensor.from_numpy(saved))
    assert_bits_equal(got.to_numpy(), want, name)


@pytest.mark.gpu
@pytest.mark.parametrize("n", SIZES)
def test_gpu_autograd_gelu(n):
    import rusttorch_b200 as rt
    _, x = _inputs(n, 40)
    assert_bits_equal(rt.autograd_gelu(rt.Tensor.from_numpy(x)).to_numpy(), O.autograd_gelu(x),
                      "autograd gelu")


@pytest.mark.gpu
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("name", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("need", [(True, True), (True, False), (False, True)])
def test_gpu_grad_binary(name, n, need):
    import rusttorch_b200 as rt
    g, a = _inputs(n, 50)
    b = O.normal(n, 52, 0, 2.0)
    b[: min(n, 3)] = [0.0, -0.0, np.inf][: min(n, 3)]
    wa, wb = O.grad_binary(name, g, a, b, *need)
    tg, ta, tb = (rt.Tensor.from_numpy(v) for v in (g, a, b))
    if name in ("add", "sub"):
        ga, gb = getattr(rt, name + "_backward")(tg, *need)
    else:
        ga, gb = getattr(rt, name + "_backward")(tg, ta, tb, *need)
    for got, want, tag in ((ga, wa, "a"), (gb, wb, "b")):
        assert (got is None) == (want is None)
        if want is not None:
            assert_bits_equal(got.to_numpy(), want, f"{name} grad_{tag}")


@pytest.mark.gpu
def test_gpu_backward_unaligned_views_and_in_place():
    import rusttorch_b200 as rt
    n = 100_003
    g, a = _inputs(n + 1, 60)
    b = O.normal(n + 1, 62)
    tg, ta, tb = (rt.Tensor.from_numpy(v) for v in (g, a, b))
    # views one element in: pointers 4 bytes off 16-byte alignment
    vg, va, vb = (rt.Tensor.from_device_ptr(t.ptr + 4, [n], owner=t) for t in (tg, ta, tb))
    wa, wb = O.grad_binary("div", g[1:].copy(), a[1:].copy(), b[1:].copy())
    ga, gb = rt.div_backward(vg, va, vb)
    assert_bits_equal(ga.to_numpy(), wa, "unaligned div a")
    assert_bits_equal(gb.to_numpy(), wb, "unaligned div b")
    # in place: grad_input written over grad_output
    want = O.grad_unary("relu", g, a)
    N.check(N.lib().rtc_relu_backward(tg.desc, ta.desc, tg.desc))
    assert_bits_equal(tg.to_numpy(), want, "relu in place")


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [[1], [4], [1000, 33], [(1 << 22) + 1]])
@pytest.mark.parametrize("mean", [False, True])
def test_gpu_sum_mean_backward(shape, mean):
    import rusttorch_b200 as rt
    for gv in (1.0, -0.0, 3.1415927, 1e-30, np.nan):
        go = rt.Tensor.from_numpy(np.array([gv], F))
        got = (rt.mean_backward if mean else rt.sum_backward)(go, shape).to_numpy()
        assert_bits_equal(got, O.fill_backward(F(gv), tuple(shape), mean), f"{shape} {gv}")


BA_CASES = [
    ((64, 96), (1, 96), (64, 96)),          # Linear bias [1, out]
    ((64, 96), (96,), (64, 96)),            # 1-D bias: generic fold
    ((64, 96), (64, 1), (64, 96)),          # row sums, one chain per row
    ((64, 1), (1, 96), (64, 96)),
    ((4, 5, 96), (96,), (4, 5, 96)),
    ((4, 1, 12), (4, 5, 12), (4, 5, 12)),   # the generic fold's own order
    ((1,), (33, 17), (33, 17)),             # one element: one chain over all
    ((8192, 4), (8192, 1), (8192, 4)),
    ((4096, 4096), (4096,), (4096, 4096)),
    ((2048, 4096), (2048, 1), (2048, 4096)),
    ((300, 33), (300, 1), (300, 33)),       # rows of 33: the unaligned chain
    ((1000, 37), (1, 37), (1000, 37)),
    ((19236, 1), (1, 1), (19236, 1)),       # [1, C] column sums with C == 1: one chain
    ((1, 1), (99, 1), (99, 1)),
    ((1 << 19, 1), (1, 1), (1 << 19, 1)),   # a long single column: the ordered-sum kernels
    ((1,), (1 << 19,), (1 << 19,)),         # one chain over all, long
]


@pytest.mark.gpu
@pytest.mark.parametrize("sa,sb,so", BA_CASES)
def test_gpu_broadcast_add_backward(sa, sb, so):
    import rusttorch_b200 as rt
    grad = O.normal(int(np.prod(so)), 70, 0, 1.0).reshape(so)
    grad.ravel()[:5] = [-0.0, -0.0, np.nan, 1e-45, -3e38][: min(5, grad.size)]
    tg = rt.Tensor.from_numpy(grad)
    ga, gb = rt.broadcast_add_backward(tg, sa, sb)
    for got, shape in ((ga, sa), (gb, sb)):
        rc, want = O.reduce_to_shape(grad, shape)
        assert rc == 0
        assert_bits_equal(got.to_numpy(), want, f"{so} -> {shape}")


@pytest.mark.gpu
def test_gpu_backward_on_host_memory():
    n = 40_000_003                     # several pipeline chunks, ragged end
    g, a = _inputs(n, 80)
    b = O.normal(n, 82)
    ga, gb = np.empty_like(g), np.empty_like(g)

    def hd(x):
        return N.Desc(x.ctypes.data, x.shape, N.F32, -1)

    dg, da, db, dga, dgb = hd(g), hd(a), hd(b), hd(ga), hd(gb)
    N.check(N.lib().rtc_mul_backward(dg.ref, da.ref, db.ref, dga.ref, dgb.ref))
    wa, wb = O.grad_binary("mul", g, a, b)
    assert_bits_equal(ga, wa, "host mul a")
    assert_bits_equal(gb, wb, "host mul b")
    y = O.unary("tanh", a)
    dy = hd(y)
    N.check(N.lib().rtc_tanh_backward(dg.ref, dy.ref, dga.ref))
    assert_bits_equal(ga, O.grad_unary("tanh", g, y), "host tanh")
