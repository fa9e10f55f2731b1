"""Ops on tensors in host memory (rtc_tensor.device == RTC_HOST_MEMORY).

The library streams host data through the current GPU in chunks with the
copies overlapped; results must be the same bits as the device path and the
oracle.  Sizes are chosen to span several chunks (a pipeline slot holds about
64 MB) and to leave ragged last chunks.
"""
import ctypes

import numpy as np
import pytest

from rusttorch_b200 import _native as N
from tests import _oracle as O
from tests.test_parity_gpu import assert_bits_equal

# Bit-exact comparisons of the transcendental activations and softmax need
# the exact math mode (the tolerance mode is tests/test_tolerance_gpu.py).
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_math")]
HOST = -1


def hdesc(a):
    return N.Desc(a.ctypes.data, a.shape, N.F32, HOST)


def pinned(n):
    p = ctypes.c_void_p()
    N.check(N.lib().rtc_host_alloc(n * 4, ctypes.byref(p)))
    arr = np.ctypeslib.as_array((ctypes.c_float * n).from_address(p.value))
    return arr, p


@pytest.mark.parametrize("n", [1, 1000, (1 << 24) + 7, 50_000_003])
def test_host_add_mul_scalar(n):
    a, b = O.uniform(n, 1), O.uniform(n, 101)
    out = np.empty_like(a)
    N.check(N.lib().rtc_add_mul_scalar(hdesc(a).ref, hdesc(b).ref, 0.5, hdesc(out).ref))
    assert_bits_equal(out, O.scalar_op("mul_scalar", O.binary("add", a, b), 0.5), "host add")


def test_host_activation_pinned_and_in_place():
    n = 30_000_001
    x, handle = pinned(n)
    try:
        x[:] = O.normal(n, 4, 0.0, 2.0)
        want = O.unary("gelu", np.ascontiguousarray(x))
        d = hdesc(x)
        N.check(N.lib().rtc_gelu(d.ref, d.ref))     # in place
        assert_bits_equal(x, want, "host gelu in place")
    finally:
        N.check(N.lib().rtc_host_free(handle))


def test_host_softmax_rows_and_middle_dim():
    x = O.normal(20000 * 1000, 4, 0.0, 2.0).reshape(20000, 1000)
    out = np.empty_like(x)
    N.check(N.lib().rtc_softmax(hdesc(x).ref, 1, hdesc(out).ref))
    assert_bits_equal(out, O.softmax(x, 1), "host softmax dim 1")
    y = O.normal(3 * 50 * 7, 5).reshape(3, 50, 7)
    out = np.empty_like(y)
    N.check(N.lib().rtc_softmax(hdesc(y).ref, 1, hdesc(out).ref))
    assert_bits_equal(out, O.softmax(y, 1), "host softmax middle dim")


@pytest.mark.parametrize("op", ["sum", "max", "mean"])
def test_host_dim_reductions(op):
    x = O.uniform(3000 * 7000, 3).reshape(3000, 7000)
    for dim in (0, 1):
        out = np.empty([d for i, d in enumerate(x.shape) if i != dim], dtype=np.float32)
        N.check(getattr(N.lib(), f"rtc_{op}_dim")(hdesc(x).ref, dim, hdesc(out).ref))
        assert_bits_equal(out, O.reduce_dim(op, x, dim), f"host {op}_dim {dim}")


def test_host_global_reductions_across_chunks():
    n = 60_000_007                       # several 16M-element chunks
    x = O.normal(n, 2)
    x[17_000_000] = np.nan               # a NaN in the second chunk
    x[40_000_000:] = -np.abs(x[40_000_000:])
    x[45_000_000] = 0.0
    x[50_000_000] = -0.0
    v = ctypes.c_double()
    for op in ("max", "min"):
        N.check(getattr(N.lib(), f"rtc_{op}")(hdesc(x).ref, ctypes.byref(v)))
        want = O.scalar_reduce(op, x)[1]
        assert np.float32(v.value).view(np.uint32) == np.float32(want).view(np.uint32), op
    y = O.normal(n, 3)
    N.check(N.lib().rtc_sum(hdesc(y).ref, ctypes.byref(v)))
    assert abs(v.value - O.sum(y)) <= 1e-6 * float(np.abs(y.astype(np.float64)).sum())


def test_host_shard_summary_matches_device_summary():
    x = O.normal(40_000_001, 6)
    x[33_000_000] = np.nan
    hs, ds = N.ShardSummary(), N.ShardSummary()
    N.check(N.lib().rtc_shard_summary_local(hdesc(x).ref, ctypes.byref(hs)))
    import rusttorch_b200 as rt
    d = rt.Tensor.from_numpy(x)
    N.check(N.lib().rtc_shard_summary_local(d.desc, ctypes.byref(ds)))
    assert hs.count == ds.count and hs.max_kind == ds.max_kind == 2
    assert hs.first_nan == ds.first_nan
    assert np.float32(hs.max).view(np.uint32) == np.float32(ds.max).view(np.uint32)
    assert np.float32(hs.min_nonnan).view(np.uint32) == np.float32(ds.min_nonnan).view(np.uint32)


def test_host_adamw_in_place():
    n = 20_000_003
    p = O.normal(n, 51, 0, 0.02)
    g = O.normal(n, 52, 0, 1e-2)
    m = O.normal(n, 53, 0, 1e-3)
    v = O.uniform(n, 54, 0.0, 1e-4)
    rc, wp, wm, wv = O.adamw(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
    dp, dg, dm, dv = hdesc(p), hdesc(g), hdesc(m), hdesc(v)
    N.check(N.lib().rtc_adamw_update(dp.ref, dg.ref, dm.ref, dv.ref, 1e-3, 0.9, 0.999, 1e-8,
                                     0.01, 10, dp.ref, dm.ref, dv.ref))
    assert_bits_equal(p, wp, "host adamw p")
    assert_bits_equal(m, wm, "host adamw m")
    assert_bits_equal(v, wv, "host adamw v")


def test_sum_device_matches_sum():
    import rusttorch_b200 as rt
    x = O.normal((1 << 22) + 3, 8)
    d = rt.Tensor.from_numpy(x)
    out = rt.Tensor([2])
    N.check(N.lib().rtc_sum_device(d.desc, ctypes.c_void_p(out.ptr)))
    got = np.empty(1, np.float64)
    rt.synchronize()
    N.check(N.lib().rtc_memcpy_d2h(0, got.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(out.ptr), 8))
    assert got[0] == rt.sum(d)
