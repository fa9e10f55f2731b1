"""Loss functions (ops/loss.rs).

CPU: the oracle against the reference's own unit tests (loss.rs:393-491) and
an independent numpy restatement; the C ABI's argument checks in the
reference's order.  GPU: the CUDA path against the oracle -- mse, l1 and
smooth_l1 bit for bit (the f64 result is identical), bce and ce within
1e-6 relative (they use a correctly rounded logf, which differs from glibc's
in the last bit for about 0.02% of inputs).
"""
import ctypes
import math

import numpy as np
import pytest

from rusttorch_b200 import _native as N
from tests import _oracle as O

F = np.float32


def a(*v):
    return np.array(v, F)


# ---- CPU: the reference's tests, through the oracle ------------------------
def test_oracle_reference_loss_kats():
    # test_mse_loss / test_mse_loss_nonzero (:398-414)
    assert abs(O.loss("mse", a(1, 2, 3, 4), a(1, 2, 3, 4))) < 1e-6
    assert abs(O.loss("mse", a(1, 2, 3), a(2, 2, 2)) - 0.6667) < 0.001
    # test_l1_loss (:417-424)
    assert abs(O.loss("l1", a(1, 2, 3), a(2, 2, 2)) - 0.6667) < 0.001
    # test_smooth_l1_loss (:427-438)
    assert abs(O.loss("smooth_l1", a(0, 2, 5), a(0, 0, 0), 1.0) - 2.0) < 0.001
    # test_binary_cross_entropy / test_cross_entropy (:441-457)
    v = O.loss("bce", a(0.9, 0.1, 0.8, 0.2), a(1, 0, 1, 0), 1e-7)
    assert 0.0 < v < 0.5
    assert O.loss("ce", a(0.7, 0.3, 0.4, 0.6), a(1, 0, 0, 1), 1e-7) > 0.0


def _unrolled(terms):
    p = [F(0)] * 8
    k = 0
    while len(terms) - k >= 8:
        for j in range(8):
            p[j] = F(p[j] + terms[k + j])
        k += 8
    acc = F(0)
    for j in range(4):
        acc = F(acc + F(p[j] + p[j + 4]))
    for v in terms[k:]:
        acc = F(acc + v)
    return acc


def test_oracle_losses_match_numpy_restatement():
    n = 1003
    pr = O.normal(n, 1, 0, 2.0)
    tg = O.normal(n, 2, 0, 2.0)
    d = (pr - tg).astype(F)
    assert O.loss("mse", pr, tg) == float(_unrolled(list((d * d).astype(F)))) / n
    assert O.loss("l1", pr, tg) == float(_unrolled(list(np.abs(d)))) / n
    b = F(0.75)
    sl = [F(F(F(F(0.5) * x) * x) / b) if abs(x) < b else F(abs(x) - F(F(0.5) * b)) for x in d]
    assert O.loss("smooth_l1", pr, tg, 0.75) == float(_unrolled(sl)) / n
    # bce / ce: one chain from -0.0, logs in double rounded to f32 (glibc's
    # logf is within 1 ulp of that), so compare within a tight tolerance
    p01 = O.uniform(n, 3, 0.0, 1.0)
    t01 = (O.uniform(n, 4, 0.0, 1.0) > 0.5).astype(F)
    eps = F(1e-7)
    acc = F(-0.0)
    for pv, tv in zip(p01, t01):
        pc = min(max(pv, eps), F(F(1) - eps))
        term = -F(F(tv * F(math.log(float(pc)))) +
                  F(F(F(1) - tv) * F(math.log(float(F(F(1) - pc))))))
        acc = F(acc + term)
    assert math.isclose(O.loss("bce", p01, t01, 1e-7), float(acc) / n, rel_tol=1e-6)


# ---- CPU: C ABI argument checks (no device work) ---------------------------
def _desc(shape, dtype=N.F32, device=0):
    return N.Desc(0x1000, shape, dtype, device)


def _err(res):
    assert not res.success
    msg = ctypes.string_at(res.error_msg).decode()
    N.lib().rtc_free_error_message(res.error_msg)
    return res.code, msg


def test_abi_loss_checks_follow_the_reference():
    L = N.lib()
    v = ctypes.c_double()
    p2, t3 = _desc([2]), _desc([3])
    # test_mse_shape_mismatch (:460-470): expected = targets' shape
    assert _err(L.rtc_mse_loss(p2.ref, t3.ref, ctypes.byref(v))) == (
        N.SHAPE_MISMATCH, "Shape mismatch in mse_loss: expected [3], got [2]")
    # test_mse_dtype_mismatch (:473-482)
    p, t64 = _desc([2, 2]), _desc([2, 2], N.F64)
    assert _err(L.rtc_mse_loss(p.ref, t64.ref, ctypes.byref(v))) == (
        N.DTYPE_MISMATCH, "Data type mismatch in mse_loss: expected float64, got float32")
    # test_mse_empty_tensor (:485-490)
    e0 = _desc([0])
    assert _err(L.rtc_mse_loss(e0.ref, e0.ref, ctypes.byref(v)))[0] == N.EMPTY_TENSOR
    # beta is checked after dtype, before emptiness
    assert _err(L.rtc_smooth_l1_loss(e0.ref, e0.ref, 0.0, ctypes.byref(v))) == (
        N.INVALID_ARGUMENT, "Invalid argument 'beta': must be positive, got 0")
    # epsilon in (0, 1); bce/ce have no separate dtype check
    assert _err(L.rtc_binary_cross_entropy_loss(p.ref, p.ref, 1.0, ctypes.byref(v))) == (
        N.INVALID_ARGUMENT, "Invalid argument 'epsilon': must be in (0, 1), got 1")
    code, msg = _err(L.rtc_cross_entropy_loss(p.ref, t64.ref, 0.5, ctypes.byref(v)))
    assert code == N.DTYPE_MISMATCH and msg == (
        "Data type mismatch in cross_entropy_loss (only floating-point supported): "
        "expected float32 or float64, got float32")
    i32 = _desc([2, 2], N.I32)
    code, msg = _err(L.rtc_l1_loss(i32.ref, i32.ref, ctypes.byref(v)))
    assert code == N.DTYPE_MISMATCH and "(only floating-point supported)" in msg


# ---- GPU ------------------------------------------------------------------
def _pair(n, seed, kind):
    if kind in ("bce", "ce"):
        p = O.uniform(n, seed, -0.1, 1.1)                    # some clamped at both ends
        t = (O.uniform(n, seed + 1, 0.0, 1.0) > 0.5).astype(F)
        if kind == "ce":
            t = O.uniform(n, seed + 1, 0.0, 1.0)
    else:
        p, t = O.normal(n, seed, 0, 2.0), O.normal(n, seed + 1, 0, 2.0)
    return p, t


PARAM = {"mse": (), "l1": (), "smooth_l1": (0.75,), "bce": (1e-7,), "ce": (1e-3,)}
API = {"mse": "mse_loss", "l1": "l1_loss", "smooth_l1": "smooth_l1_loss",
       "bce": "binary_cross_entropy_loss", "ce": "cross_entropy_loss"}


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 7, 8, 9, 1003, 2048 * 8 + 5, (1 << 20) + 3])
@pytest.mark.parametrize("kind", list(PARAM))
def test_gpu_losses(kind, n):
    import rusttorch_b200 as rt
    p, t = _pair(n, 10, kind)
    want = O.loss(kind, p, t, *PARAM[kind])
    got = getattr(rt, API[kind])(rt.Tensor.from_numpy(p), rt.Tensor.from_numpy(t), *PARAM[kind])
    if kind in ("bce", "ce"):
        assert math.isclose(got, want, rel_tol=1e-6, abs_tol=1e-12), (got, want)
    else:
        assert got == want or (math.isnan(got) and math.isnan(want)), (got, want)


@pytest.mark.gpu
def test_gpu_mse_full_cfg1_size_and_specials():
    import rusttorch_b200 as rt
    n = 1 << 24
    p, t = O.normal(n, 20), O.normal(n, 21)
    want = O.loss("mse", p, t)
    assert rt.mse_loss(rt.Tensor.from_numpy(p), rt.Tensor.from_numpy(t)) == want
    p[5], t[9] = np.inf, np.nan
    for kind in ("mse", "l1", "smooth_l1"):
        got = getattr(rt, API[kind])(rt.Tensor.from_numpy(p[:4099]),
                                     rt.Tensor.from_numpy(t[:4099]), *PARAM[kind])
        assert math.isnan(got) and math.isnan(O.loss(kind, p[:4099], t[:4099], *PARAM[kind]))
