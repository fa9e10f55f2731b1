"""Rows beyond the core path: broadcasting binary ops (ops/broadcast.rs) and
the nn optimizers (nn/optim.rs).  CPU: the oracle against independent numpy
restatements and the C ABI's validation; GPU: the CUDA path against the
oracle, bit for bit."""
import ctypes

import numpy as np
import pytest

from rusttorch_b200 import _native as N
from tests import _oracle as O

F = np.float32
BCAST = [((4, 5), (5,)), ((4, 1), (1, 6)), ((3, 1, 7), (2, 1)), ((2, 3, 4), (2, 3, 4)),
         ((1,), (9, 3)), ((), (3, 2)), ((65, 130), (65, 1)), ((8, 1, 33), (8, 17, 1))]


def bits(x):
    return np.asarray(x, dtype=F).view(np.uint32)


# ---- CPU: oracle pins ---------------------------------------------------
@pytest.mark.parametrize("sa,sb", BCAST)
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_oracle_broadcast_matches_numpy(sa, sb, op):
    a = O.normal(int(np.prod(sa)), 3).reshape(sa)
    b = O.normal(int(np.prod(sb)), 4).reshape(sb)
    if op == "div":
        b = np.where(b == 0, F(0.5), b).astype(F)
    rc, out = O.broadcast(op, np.ascontiguousarray(a), np.ascontiguousarray(b))
    assert rc == 0
    want = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[op](a, b)
    np.testing.assert_array_equal(bits(out), bits(want.astype(F)))


def test_oracle_broadcast_rejects_incompatible():
    rc, _ = O.broadcast("add", np.ones((2, 3), F), np.ones((4,), F))
    assert rc == 9


def test_oracle_nn_adam_matches_python_restatement():
    n = 257
    p, g = O.normal(n, 1, 0, 0.5), O.normal(n, 2, 0, 0.1)
    m, v = O.normal(n, 3, 0, 0.01), O.uniform(n, 4, 0.0, 1e-3)
    lr, b1, b2, eps, t = F(1e-3), F(0.9), F(0.999), F(1e-8), 7
    po, mo, vo = O.nn_adam(p, g, m, v, lr, b1, b2, eps, t)
    import math
    bc1 = F(1.0) - F(math.pow(float(b1), float(F(t))))   # glibc powf is within 1 ulp of this
    bc2 = F(1.0) - F(math.pow(float(b2), float(F(t))))
    for j in range(n):
        nm = F(F(b1 * m[j]) + F(F(F(1) - b1) * g[j]))
        nv = F(F(b2 * v[j]) + F(F(F(F(1) - b2) * g[j]) * g[j]))
        assert bits(mo[j]) == bits(nm) and bits(vo[j]) == bits(nv)
        want = F(p[j] - F(F(lr * F(nm / bc1)) / F(F(np.sqrt(F(nv / bc2))) + eps)))
        assert abs(float(po[j]) - float(want)) <= 2e-7 * max(1.0, abs(float(want)))


def test_oracle_nn_sgd_matches_python_restatement():
    n = 100
    p, g, vel = O.normal(n, 5), O.normal(n, 6), O.normal(n, 7)
    po, vo = O.nn_sgd(p, g, vel, F(0.1), F(0.9), F(5e-4))
    want_v = (F(F(F(0.9) * vel) + g) + F(F(5e-4) * p)).astype(F)
    np.testing.assert_array_equal(bits(vo), bits(want_v))
    np.testing.assert_array_equal(bits(po), bits((p - F(0.1) * want_v).astype(F)))
    po, _ = O.nn_sgd(p, g, None, F(0.1), F(0.0), F(5e-4))
    np.testing.assert_array_equal(bits(po), bits((p - F(0.1) * (g + F(5e-4) * p)).astype(F)))


# ---- CPU: C ABI validation (no device work) -----------------------------
def _desc(shape, dtype=N.F32):
    return N.Desc(0x1000, shape, dtype, 0)


def _err(res):
    assert not res.success
    msg = ctypes.string_at(res.error_msg).decode()
    N.lib().rtc_free_error_message(res.error_msg)
    return res.code, msg


def test_broadcast_errors_follow_the_reference():
    a, b, o = _desc([2, 3]), _desc([4]), _desc([2, 3])
    assert _err(N.lib().rtc_add_broadcast(a.ref, b.ref, o.ref)) == (
        N.BROADCAST_ERROR, "Cannot broadcast shapes [2, 3] and [4]: Incompatible shapes for "
        "broadcasting")
    b64 = _desc([3], N.F64)
    assert _err(N.lib().rtc_mul_broadcast(a.ref, b64.ref, o.ref)) == (
        N.DTYPE_MISMATCH, "Data type mismatch in broadcast_tensors: expected float32, got float64")
    i1, i2, io = _desc([2, 3], N.I32), _desc([3], N.I32), _desc([2, 3], N.I32)
    assert _err(N.lib().rtc_div_broadcast(i1.ref, i2.ref, io.ref)) == (
        N.INVALID_ARGUMENT, "Invalid argument 'dtype': Division requires floating-point tensors")


def test_nn_sgd_counts_elements():
    p, g = _desc([2, 3]), _desc([7])
    code, msg = _err(N.lib().rtc_nn_sgd_step(p.ref, g.ref, None, 0.1, 0.0, 0.0, p.ref, None))
    assert code == N.SHAPE_MISMATCH and "SGD step" in msg


# ---- GPU ------------------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("sa,sb", BCAST + [((4096, 4096), (4096,)), ((1024, 1), (1024, 2048)),
                                           ((2048,), (64, 2048)), ((300, 1), (1, 8)),
                                           ((64, 256), (64, 1))])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_gpu_broadcast(sa, sb, op):
    import rusttorch_b200 as rt
    a = O.normal(int(np.prod(sa)), 3).reshape(sa)
    b = O.normal(int(np.prod(sb)), 4).reshape(sb)
    rc, want = O.broadcast(op, np.ascontiguousarray(a), np.ascontiguousarray(b))
    got = getattr(rt, op + "_broadcast")(rt.Tensor.from_numpy(a), rt.Tensor.from_numpy(b))
    assert got.shape() == list(want.shape)
    g = got.to_numpy()
    same = (bits(g) == bits(want)) | (np.isnan(g) & np.isnan(want))
    assert same.all()


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 1001, 1 << 22])
def test_gpu_nn_adam_and_sgd(n):
    import rusttorch_b200 as rt
    p, g = O.normal(n, 1, 0, 0.5), O.normal(n, 2, 0, 0.1)
    m, v = O.normal(n, 3, 0, 0.01), O.uniform(n, 4, 0.0, 1e-3)
    for t in (1, 10):
        wp, wm, wv = O.nn_adam(p, g, m, v, F(1e-3), F(0.9), F(0.999), F(1e-8), t)
        po, mo, vo = rt.nn_adam_step(*(rt.Tensor.from_numpy(x) for x in (p, g, m, v)),
                                     1e-3, 0.9, 0.999, 1e-8, t)
        for got, want in ((po, wp), (mo, wm), (vo, wv)):
            np.testing.assert_array_equal(bits(got.to_numpy()), bits(want))
    for mom, wd in ((0.0, 0.0), (0.0, 5e-4), (0.9, 5e-4)):
        wp, wv = O.nn_sgd(p, g, m, F(0.05), F(mom), F(wd))
        po, vo = rt.nn_sgd_step(rt.Tensor.from_numpy(p), rt.Tensor.from_numpy(g),
                                rt.Tensor.from_numpy(m), 0.05, mom, wd)
        np.testing.assert_array_equal(bits(po.to_numpy()), bits(wp))
        if mom > 0:
            np.testing.assert_array_equal(bits(vo.to_numpy()), bits(wv))
