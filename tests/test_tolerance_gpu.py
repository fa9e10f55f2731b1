"""The tolerance math mode on the GPU (the library's default).

Each transcendental activation and softmax must be within north_star's
tolerance of the oracle (the reference's formula over glibc): 1e-6 relative
error or 4 ulp, NaN where the reference gives NaN.  The device results must
also equal the host build of the same rules (tests/native/fastmath_check.cpp)
bit for bit: that is what carries the host's check of all 2^32 inputs
(tests/test_fastmath.py) over to the GPU.
"""
import ctypes

import numpy as np
import pytest

import rusttorch_b200 as rt
from rusttorch_b200 import _native as N
from tests import _oracle as O
from tests.test_fastmath import OPS, load_fastmath_lib, ordered

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def tolerance_math():
    lib = N.lib()
    before = lib.rtc_get_math_mode()
    N.check(lib.rtc_set_math_mode(N.MATH_TOLERANCE))
    yield
    N.check(lib.rtc_set_math_mode(before))


@pytest.fixture(scope="module")
def fm():
    return load_fastmath_lib()


def dev(a):
    return rt.Tensor.from_numpy(np.ascontiguousarray(a, dtype=np.float32))


def bit_sweep(stride=257, offset=0):
    u = np.arange(offset, 1 << 32, stride, dtype=np.uint64).astype(np.uint32)
    return u.view(np.float32)


def assert_bits_equal(got, want, what):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    if not same.all():
        i = np.flatnonzero(~same.ravel())[:5]
        raise AssertionError(f"{what}: {(~same).sum()} differ; first at {i}: "
                             f"got {got.ravel()[i]} want {want.ravel()[i]}")


def assert_within_tolerance(got, want, what):
    """north_star: within 1e-6 relative error, or 4 ulp (NaN equals NaN)."""
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    nan_g, nan_w = np.isnan(got), np.isnan(want)
    assert (nan_g == nan_w).all(), (what, "NaN mismatch", np.flatnonzero(nan_g != nan_w)[:5])
    g, w = got[~nan_w], want[~nan_w]
    ulps = np.abs(ordered(g) - ordered(w))
    with np.errstate(invalid="ignore", divide="ignore"):
        rel = np.where(g == w, 0.0, np.abs(g.astype(np.float64) - w) / np.abs(w.astype(np.float64)))
    bad = (ulps > 4) & (rel > 1e-6)
    if bad.any():
        i = np.flatnonzero(bad)[:5]
        raise AssertionError(f"{what}: {bad.sum()} outside 1e-6 rel / 4 ulp; got {g[i]} want "
                             f"{w[i]} rel {rel[i]}")


def host_rule(fm, op, x):
    out = np.empty_like(x)
    fm.fm_eval(OPS[op], x.ctypes.data, out.ctypes.data, x.size)
    return out


ACTS = ["sigmoid", "swish", "tanh", "softplus", "mish", "gelu"]


@pytest.mark.parametrize("op", ACTS)
def test_activation_bit_sweep(fm, op):
    """Every 257th float bit pattern (all exponents, signs, subnormals,
    infinities, NaNs): equal to the host build, within tolerance of the
    oracle."""
    x = bit_sweep(257)
    got = getattr(rt, op)(dev(x)).to_numpy()
    assert_bits_equal(got, host_rule(fm, op, x), f"{op} vs its host build")
    assert_within_tolerance(got, O.unary(op, x), f"{op} vs oracle")


@pytest.mark.parametrize("op", ACTS)
def test_cfg4_full_size(fm, op):
    x = O.normal(32768 * 4096, 4, 0.0, 2.0).reshape(32768, 4096)
    got = getattr(rt, op)(dev(x)).to_numpy()
    assert_within_tolerance(got, O.unary(op, x), f"{op} cfg4")
    if op == "gelu":
        assert_bits_equal(got, host_rule(fm, op, x.ravel()).reshape(x.shape), "gelu cfg4 host")


@pytest.mark.parametrize("lo,hi", [(-6.0, -1.0), (-1.5, 3.0), (0.0, 8.0), (-12.0, -8.0)])
@pytest.mark.parametrize("n", [1, 7, 4096 + 3, 1 << 20])
def test_gelu_split_queue(fm, lo, hi, n):
    """GELU's split kernel with every element queued for the exact tanh,
    none, or a mix; ragged tails; and the scalar path for misaligned data."""
    x = O.uniform(n + 1, 61, lo, hi)
    got = rt.gelu(dev(x[:n])).to_numpy()
    assert_bits_equal(got, host_rule(fm, "gelu", x[:n]), f"gelu [{lo},{hi}) n={n}")
    t = dev(x)
    out = rt.Tensor.from_numpy(np.zeros(n + 1, np.float32))
    va = rt.Tensor.from_device_ptr(t.ptr + 4, [n], owner=t)
    vo = rt.Tensor.from_device_ptr(out.ptr + 4, [n], owner=out)
    N.check(N.lib().rtc_gelu(va.desc, vo.desc))
    assert_bits_equal(vo.to_numpy(), host_rule(fm, "gelu", x[1:]), f"misaligned gelu n={n}")


def test_softmax_cfg4_full_size(fm):
    x = O.normal(32768 * 4096, 4, 0.0, 2.0).reshape(32768, 4096)
    got = rt.softmax(dev(x), 1).to_numpy()
    assert_within_tolerance(got, O.softmax(x, 1), "softmax cfg4")
    host = np.empty_like(x)
    fm.fm_softmax_rows.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                   ctypes.c_void_p, ctypes.c_int]
    fm.fm_softmax_rows(x.ctypes.data, 32768, 4096, host.ctypes.data, 16)
    assert_bits_equal(got, host, "softmax cfg4 vs its host build")


@pytest.mark.parametrize("shape,dim,std", [((3, 5), 1, 3), ((7, 1000), 1, 10), ((50, 6), 0, 3),
                                           ((4, 5, 6), 1, 3), ((2, 70001), 1, 3),
                                           ((6, 4097), 1, 0.1), ((3, 8196), 1, 3),
                                           ((4099, 1), 0, 3), ((512, 4096), 1, 30)])
def test_softmax_shapes(shape, dim, std):
    x = O.normal(int(np.prod(shape)), 42, 0, std).reshape(shape)
    assert_within_tolerance(rt.softmax(dev(x), dim).to_numpy(), O.softmax(x, dim),
                            f"softmax {shape} {dim}")


def test_softmax_special_rows():
    x = O.normal(8 * 64, 43).reshape(8, 64)
    x[1, 5] = np.nan
    x[2, :] = -np.inf
    x[3, 7] = np.inf
    x[4, :] = 0.0
    x[5, :] = 1e30
    x[6, :] = -200.0
    x[6, 0] = 0.0
    assert_within_tolerance(rt.softmax(dev(x), 1).to_numpy(), O.softmax(x, 1), "softmax specials")


def test_primitives_match_their_host_build(fm):
    lib = N.lib()
    x = bit_sweep(61)
    d = dev(x)
    out = rt.Tensor.from_numpy(np.zeros_like(x))
    for which, op in ((0, "exp"), (2, "tanh")):
        N.check(lib.rtc_selftest_fastmath(which, ctypes.c_void_p(d.ptr), ctypes.c_void_p(out.ptr),
                                          x.size))
        assert_bits_equal(out.to_numpy(), host_rule(fm, op, x), op)
    pos = x[(x > 1.17549435e-38) & (x < np.inf)]
    dp, op_ = dev(pos), rt.Tensor.from_numpy(np.zeros_like(pos))
    N.check(lib.rtc_selftest_fastmath(1, ctypes.c_void_p(dp.ptr), ctypes.c_void_p(op_.ptr),
                                      pos.size))
    assert_bits_equal(op_.to_numpy(), host_rule(fm, "log", pos), "log")


def test_reciprocal_is_correctly_rounded():
    """rcp_cr against IEEE division: every float in [1, 2) and a stride
    through [2, 2^64]."""
    lib = N.lib()
    one = np.arange(0x3f800000, 0x40000000, dtype=np.uint32).view(np.float32)
    rest = np.arange(0x40000000, 0x5f800001, 7, dtype=np.uint32).view(np.float32)
    for x in (one, rest):
        d, out = dev(x), rt.Tensor.from_numpy(np.zeros_like(x))
        N.check(lib.rtc_selftest_fastmath(3, ctypes.c_void_p(d.ptr), ctypes.c_void_p(out.ptr),
                                          x.size))
        assert_bits_equal(out.to_numpy(), np.float32(1.0) / x, "rcp_cr")


def test_mode_switch_changes_only_the_math():
    """The same input through both modes: exact is glibc's bits, tolerance is
    within tolerance of them."""
    lib = N.lib()
    x = O.normal(1 << 16, 44, 0, 3)
    try:
        N.check(lib.rtc_set_math_mode(N.MATH_EXACT))
        for op in ("sigmoid", "tanh", "gelu", "swish"):
            assert_bits_equal(getattr(rt, op)(dev(x)).to_numpy(), O.unary(op, x), f"exact {op}")
        assert_bits_equal(rt.softmax(dev(x.reshape(16, 4096)), 1).to_numpy(),
                          O.softmax(x.reshape(16, 4096), 1), "exact softmax")
    finally:
        N.check(lib.rtc_set_math_mode(N.MATH_TOLERANCE))
    for op in ("sigmoid", "tanh", "gelu", "swish"):
        assert_within_tolerance(getattr(rt, op)(dev(x)).to_numpy(), O.unary(op, x), f"tol {op}")
