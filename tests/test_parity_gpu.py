"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Inputs come from the oracle's seeded generator with BASELINE.json's shapes
and distributions, are copied to the GPU, run through librusttorch_cuda.so,
and the results are compared with the oracle on the same inputs:
  * bit-exact (NaN compares equal to NaN): add/sub/mul/div, scalar ops, fma,
    relu/leaky_relu, max/min, the dim reductions, AdamW/Adam/SGD, and — since
    the device restates glibc's expf/tanhf — sigmoid, tanh, GELU, SiLU, ELU,
    SELU, softsign and softmax;
  * |sum - ref| <= 1e-6 * sum|x| for sum and mean (BASELINE.json tolerance);
  * softplus and mish, whose log is rounded from double rather than taken
    from glibc's table-driven logf: bit-exact with the same rule built for
    the host, and within 1 ulp (softplus) / 6 ulp (mish) of the oracle.
"""
import ctypes

import numpy as np
import pytest

import rusttorch_b200 as rt
from rusttorch_b200 import _native as N
from tests import _oracle as O

# Bit-exact comparisons of the transcendental activations and softmax need
# the exact math mode (the tolerance mode is tests/test_tolerance_gpu.py).
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_math")]

NAN = np.float32(np.nan)


def bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32)


def assert_bits_equal(got, want, what=""):
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    same = (bits(got) == bits(want)) | (np.isnan(got) & np.isnan(want))
    if not same.all():
        i = np.flatnonzero(~same.ravel())[:5]
        raise AssertionError(f"{what}: {(~same).sum()} of {same.size} differ; first at {i}: "
                             f"got {got.ravel()[i]} want {want.ravel()[i]}")


def ulp_diff(a, b):
    ia = bits(a).astype(np.int64)
    ib = bits(b).astype(np.int64)
    ia = np.where(ia < 0x80000000, ia, 0x80000000 - ia)
    ib = np.where(ib < 0x80000000, ib, 0x80000000 - ib)
    return np.where(np.isnan(a) & np.isnan(b), 0, np.abs(ia - ib))


def dev(a):
    return rt.Tensor.from_numpy(np.ascontiguousarray(a, dtype=np.float32))


def edge_values():
    v = [0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-38, -1e-38, 3.4e38,
         -3.4e38, 20.0, 20.000002, -20.0, 88.72, 88.73, -103.9, -104.0, 22.0, -22.0, 1e-30, 0.5]
    return np.array(v, dtype=np.float32)


def bit_sweep(stride=257, offset=0):
    """Every stride-th float32 bit pattern: all exponents, signs, NaNs."""
    u = np.arange(offset, 1 << 32, stride, dtype=np.uint64).astype(np.uint32)
    return u.view(np.float32)


# ---------------------------------------------------------------- cfg 1
def test_cfg1_add_then_mul_scalar_full_size():
    n = 1 << 24
    a = O.uniform(n, 1)
    b = O.uniform(n, 101)
    want = O.scalar_op("mul_scalar", O.binary("add", a, b), 0.5)
    da, db = dev(a), dev(b)
    assert_bits_equal(rt.add_mul_scalar(da, db, 0.5).to_numpy(), want, "fused add->mul_scalar")
    assert_bits_equal(rt.mul_scalar(rt.add(da, db), 0.5).to_numpy(), want, "add then mul_scalar")


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_binary_ops_edge_and_random(op):
    rng = np.random.default_rng(5)
    e = edge_values()
    a = np.concatenate([np.repeat(e, e.size), O.normal(100003, 11, 0, 3)]).astype(np.float32)
    b = np.concatenate([np.tile(e, e.size), O.normal(100003, 12, 0, 3)]).astype(np.float32)
    rng.shuffle(a)
    want = O.binary(op, a, b)
    assert_bits_equal(getattr(rt, op)(dev(a), dev(b)).to_numpy(), want, op)


def test_scalar_ops_and_fma():
    x = np.concatenate([edge_values(), O.normal(65537, 13, 0, 2)])
    y = O.normal(x.size, 14)
    z = O.normal(x.size, 15)
    assert_bits_equal(rt.add_scalar(dev(x), 10.0).to_numpy(), O.scalar_op("add_scalar", x, 10.0))
    assert_bits_equal(rt.mul_scalar(dev(x), 0.5).to_numpy(), O.scalar_op("mul_scalar", x, 0.5))
    assert_bits_equal(rt.mul_scalar_simd(dev(x), -3.0).to_numpy(), O.scalar_op("mul_scalar", x, -3.0))
    assert_bits_equal(rt.fused_multiply_add(dev(x), dev(y), dev(z)).to_numpy(), O.fma(x, y, z))
    assert_bits_equal(rt.add_simd(dev(x), dev(y)).to_numpy(), O.binary("add", x, y))
    assert_bits_equal(rt.mul_simd(dev(x), dev(y)).to_numpy(), O.binary("mul", x, y))


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 255, 4097, 1000003])
def test_odd_sizes(n):
    a = O.uniform(n, 21)
    b = O.uniform(n, 22)
    assert_bits_equal(rt.add(dev(a), dev(b)).to_numpy(), O.binary("add", a, b), f"add n={n}")
    assert_bits_equal(rt.gelu(dev(a)).to_numpy(), O.unary("gelu", a), f"gelu n={n}")


def test_misaligned_pointers_take_the_scalar_path():
    n = 100001
    base_a, base_o = rt.Tensor([n + 1]), rt.Tensor([n + 1])
    a = O.uniform(n + 1, 23)
    N.check(N.lib().rtc_memcpy_h2d(0, ctypes.c_void_p(base_a.ptr), a.ctypes.data_as(ctypes.c_void_p),
                                   a.nbytes))
    va = rt.Tensor.from_device_ptr(base_a.ptr + 4, [n], owner=base_a)
    vo = rt.Tensor.from_device_ptr(base_o.ptr + 4, [n], owner=base_o)
    N.check(N.lib().rtc_sigmoid(va.desc, vo.desc))
    assert_bits_equal(vo.to_numpy(), O.unary("sigmoid", a[1:]), "misaligned sigmoid")
    N.check(N.lib().rtc_add(va.desc, va.desc, vo.desc))
    assert_bits_equal(vo.to_numpy(), O.binary("add", a[1:], a[1:]), "misaligned add")


def test_flat_f32_api():
    n = 12345
    a, b = O.uniform(n, 31), O.uniform(n, 32)
    da, db, do = dev(a), dev(b), rt.Tensor([n])
    for name, want in [("rtc_add_f32", O.binary("add", a, b)), ("rtc_mul_f32", O.binary("mul", a, b))]:
        N.check(getattr(N.lib(), name)(ctypes.c_void_p(da.ptr), ctypes.c_void_p(db.ptr),
                                       ctypes.c_void_p(do.ptr), n))
        assert_bits_equal(do.to_numpy(), want, name)
    N.check(N.lib().rtc_relu_f32(ctypes.c_void_p(da.ptr), ctypes.c_void_p(do.ptr), n))
    assert_bits_equal(do.to_numpy(), O.unary("relu", a), "relu_f32")


# ---------------------------------------------------------------- cfg 4
BIT_EXACT_UNARY = ["relu", "sigmoid", "tanh", "gelu", "swish", "selu", "softsign"]


@pytest.mark.parametrize("op", BIT_EXACT_UNARY + ["leaky_relu", "elu"])
def test_activation_bit_sweep(op):
    """A stride over all 2^32 float bit patterns (every exponent, both signs,
    subnormals, infinities, NaNs), bit-exact against glibc through the oracle."""
    x = bit_sweep(257)
    extra = {"leaky_relu": (0.01,), "elu": (1.0,)}.get(op, ())
    want = O.unary(op, x, *extra)
    got = getattr(rt, op)(dev(x), *extra).to_numpy()
    assert_bits_equal(got, want, op)


@pytest.mark.parametrize("op", ["softplus", "mish"])
def test_log_based_activations(op):
    """Bit-exact with the device rule built for the host (rt_ops.cuh under
    g++), which is within 1 ulp (softplus) and 6 ulp (mish) of the reference's
    glibc formula over all 2^32 inputs (tests/test_libm_restatement.py)."""
    from tests.test_libm_restatement import ACT_BOUND, MISH_WORST, load_check_lib
    worst = np.array(MISH_WORST, dtype=np.uint32).view(np.float32)
    x = np.concatenate([bit_sweep(1021), O.normal(1 << 20, 41, 0, 2), worst])
    x = x[np.isfinite(x)]
    which = ["softplus", "mish"].index(op)
    host = np.empty_like(x)
    load_check_lib().act_restated(which, x.ctypes.data, host.ctypes.data, x.size)
    got = getattr(rt, op)(dev(x)).to_numpy()
    assert_bits_equal(got, host, f"{op} vs its host build")
    d = ulp_diff(got, O.unary(op, x))
    assert d.max() <= ACT_BOUND[which], (op, x[d.argmax()], d.max())


@pytest.mark.parametrize("op", ["relu", "gelu", "swish", "sigmoid", "tanh"])
def test_cfg4_activations_full_size(op):
    x = O.normal(32768 * 4096, 4, 0.0, 2.0).reshape(32768, 4096)
    assert_bits_equal(getattr(rt, op)(dev(x)).to_numpy(), O.unary(op, x), op)


def test_cfg4_softmax_full_size():
    x = O.normal(32768 * 4096, 4, 0.0, 2.0).reshape(32768, 4096)
    assert_bits_equal(rt.softmax(dev(x), 1).to_numpy(), O.softmax(x, 1), "softmax cfg4")


@pytest.mark.parametrize("shape,dim", [((3, 5), 1), ((7, 1000), 1), ((50, 6), 0), ((1, 1), 0),
                                       ((4, 5, 6), 0), ((4, 5, 6), 1), ((4, 5, 6), 2),
                                       ((2, 70001), 1), ((9,), 0), ((6, 4097), 1),
                                       ((5, 12), 1), ((3, 2052), 1), ((4, 8192), 1),
                                       ((3, 8196), 1), ((2, 1024), 1)])
def test_softmax_shapes(shape, dim):
    x = O.normal(int(np.prod(shape)), 42, 0, 3).reshape(shape)
    assert_bits_equal(rt.softmax(dev(x), dim).to_numpy(), O.softmax(x, dim), f"softmax {shape} {dim}")


def test_softmax_special_rows():
    x = O.normal(8 * 64, 43).reshape(8, 64)
    x[1, 5] = np.nan
    x[2, :] = -np.inf
    x[3, 7] = np.inf
    x[4, :] = 0.0
    x[4, 3] = -0.0
    x[5, :] = 1e30
    assert_bits_equal(rt.softmax(dev(x), 1).to_numpy(), O.softmax(x, 1), "softmax specials")


@pytest.mark.parametrize("shape", [(20000, 640), (3000, 2048), (2500, 4096), (1000, 512),
                                   (999, 1028), (7, 3000)])
def test_softmax_pipelined_rows(shape):
    """Many rows at each register tier of the row kernel, with rows of NaN,
    -inf, +inf, zeros and huge values among ordinary ones."""
    rows, n = shape
    x = O.normal(rows * n, 44, 0, 3).reshape(shape)
    for r in range(0, rows, max(1, rows // 7)):
        k = (r // max(1, rows // 7)) % 5
        if k == 0:
            x[r, r % n] = np.nan
        elif k == 1:
            x[r, :] = -np.inf
        elif k == 2:
            x[r, (3 * r) % n] = np.inf
        elif k == 3:
            x[r, :] = 0.0
        else:
            x[r, :] = 1e30
    got = rt.softmax(dev(x), 1).to_numpy()
    rt.synchronize()          # raises if a kernel gave up a bounded wait
    assert_bits_equal(got, O.softmax(x, 1), f"softmax {shape}")


# ---------------------------------------------------------------- cfg 2
def _check_sum(got, x):
    want = O.sum(x)
    tol = 1e-6 * float(np.abs(x.astype(np.float64)).sum())
    assert abs(got - want) <= tol, (got, want, tol)


def test_cfg2_global_reductions_full_size():
    x = O.normal(1 << 28, 2)
    d = dev(x)
    _check_sum(rt.sum(d), x)
    assert abs(rt.mean(d) - O.scalar_reduce("mean", x)[1]) <= 1e-6 * float(np.abs(x).mean())
    assert bits(rt.max(d)) == bits(O.scalar_reduce("max", x)[1])
    assert bits(rt.min(d)) == bits(O.scalar_reduce("min", x)[1])
    s, m, mx, mn = rt.stats(d)
    _check_sum(s, x)
    assert mx == rt.max(d) and mn == rt.min(d)


REDUCE_CASES = {
    "zero_ties": np.array([-1.0, 0.0, -0.0, -2.0, 0.0, -0.0], dtype=np.float32),
    "zero_ties_rev": np.array([-0.0, -3.0, 0.0, -0.0, 0.0, -5.0], dtype=np.float32),
    "nan_middle": np.array([1.0, np.nan, 0.5, 0.25], dtype=np.float32),
    "nan_last": np.array([3.0, 1.0, np.nan], dtype=np.float32),
    "nan_first": np.array([np.nan, 1.0, 2.0], dtype=np.float32),
    "all_nan": np.array([np.nan] * 5, dtype=np.float32),
    "infs": np.array([np.inf, -np.inf, 1.0], dtype=np.float32),
    "one": np.array([7.5], dtype=np.float32),
    "neg_zero_only": np.array([-0.0], dtype=np.float32),
    "nan_then_zeros": np.array([5.0, np.nan, -0.0, -1.0, 0.0, -0.0], dtype=np.float32),
}


@pytest.mark.parametrize("name", sorted(REDUCE_CASES))
def test_global_reduction_edge_cases(name):
    x = REDUCE_CASES[name]
    d = dev(x)
    for op in ("max", "min"):
        got = getattr(rt, op)(d)
        _, want = O.scalar_reduce(op, x)
        assert (np.isnan(got) and np.isnan(want)) or bits(got) == bits(want), (name, op, got, want)
    got = rt.sum(d)
    want = O.sum(x)
    assert (np.isnan(got) and np.isnan(want)) or got == want, (name, got, want)


def test_global_reduction_large_with_planted_nans_and_zeros():
    n = (1 << 22) + 3
    x = O.normal(n, 44)
    x[123456] = np.nan
    x[3000000] = np.nan
    x[3000001:] = -np.abs(x[3000001:])
    x[3500000] = 0.0
    x[3600000] = -0.0
    d = dev(x)
    for op in ("max", "min"):
        got = getattr(rt, op)(d)
        _, want = O.scalar_reduce(op, x)
        assert bits(got) == bits(want), (op, got, want)


def test_reduction_at_misaligned_offset():
    n = 1000001
    base = dev(O.normal(n + 3, 45))
    x = O.normal(n + 3, 45)[3:]
    v = rt.Tensor.from_device_ptr(base.ptr + 12, [n], owner=base)
    _check_sum(rt.sum(v), x)
    assert bits(rt.max(v)) == bits(O.scalar_reduce("max", x)[1])


def test_sharded_stats_one_process():
    """rtc_sharded_stats over shards (on every visible GPU, round-robin) equals
    the reference's reductions of the whole tensor."""
    import torch
    ngpu = max(1, torch.cuda.device_count())
    n = 10_000_003
    x = O.normal(n, 49)
    x[4_000_000] = np.nan
    cuts = [0, 1, 2_500_000, 2_500_000, 7_000_000, n]      # includes empty shards
    shards = [rt.Tensor.from_numpy(np.ascontiguousarray(x[a:b]), device=i % ngpu)
              for i, (a, b) in enumerate(zip(cuts[:-1], cuts[1:]))]
    s, mean, mx, mn = rt.sharded_stats(shards)
    assert np.isnan(s) and np.isnan(mean)
    assert bits(np.float32(mx)) == bits(O.scalar_reduce("max", x)[1])
    assert bits(np.float32(mn)) == bits(O.scalar_reduce("min", x)[1])
    y = O.normal(n, 50)
    shards = [rt.Tensor.from_numpy(np.ascontiguousarray(y[a:b]), device=i % ngpu)
              for i, (a, b) in enumerate(zip(cuts[:-1], cuts[1:]))]
    s, mean, mx, mn = rt.sharded_stats(shards)
    _check_sum(s, y)
    assert bits(np.float32(mx)) == bits(O.scalar_reduce("max", y)[1])
    assert bits(np.float32(mn)) == bits(O.scalar_reduce("min", y)[1])


# ---------------------------------------------------------------- cfg 3
@pytest.mark.parametrize("op", ["sum", "max", "mean"])
@pytest.mark.parametrize("dim", [0, 1])
def test_cfg3_dim_reductions_full_size(op, dim):
    x = O.uniform(8192 * 16384, 3).reshape(8192, 16384)
    got = getattr(rt, f"{op}_dim")(dev(x), dim).to_numpy()
    assert_bits_equal(got, O.reduce_dim(op, x, dim), f"{op}_dim {dim}")


@pytest.mark.parametrize("shape", [(13, 37), (5, 1), (1, 5), (3, 40, 36), (2, 3, 4, 5), (17,),
                                   (6, 1003), (300, 6), (2, 129, 64), (7, 8), (5, 1004),
                                   (9, 260), (3, 4096), (1, 65536), (2, 7, 512)])
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_dim_reduction_shapes(shape, op):
    x = O.normal(int(np.prod(shape)), 46, 0, 2).reshape(shape)
    for dim in range(len(shape)):
        got = getattr(rt, f"{op}_dim")(dev(x), dim).to_numpy()
        assert_bits_equal(got, O.reduce_dim(op, x, dim), f"{op}_dim {shape} dim={dim}")


@pytest.mark.parametrize("shape,dim", [((32768, 4096), 0), ((4, 1000, 132), 1), ((3, 777, 4), 1),
                                       ((1000, 2, 8), 1), ((2049, 300), 0), ((5, 3, 4096), 1),
                                       ((1 << 20, 4), 0), ((257, 1028), 0)])
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_tma_strip_shapes(shape, dim, op):
    """Non-last-axis reductions on the TMA-staged path: ragged last tiles
    (rows and columns), several outer slices, NaN and zero columns."""
    x = O.normal(int(np.prod(shape)), 48, 0, 2).reshape(shape)
    flat = x.reshape(-1, shape[-1])
    flat[3, 1] = np.nan
    flat[:, 2] = -np.abs(flat[:, 2])
    flat[7 % flat.shape[0], 2] = 0.0
    got = getattr(rt, f"{op}_dim")(dev(x), dim).to_numpy()
    rt.synchronize()          # raises if a kernel gave up a bounded wait
    assert_bits_equal(got, O.reduce_dim(op, x, dim), f"{op}_dim {shape} dim={dim}")


@pytest.mark.parametrize("shape", [(13, 1028), (1, 1024), (1000, 2052), (7, 8196), (4099, 4096),
                                   (3, 5, 1100), (5001, 1028), (4200, 2052), (9000, 1024),
                                   (4147, 1056), (6001, 4128)])
@pytest.mark.parametrize("op", ["sum", "mean"])
def test_last_axis_sum_row_kernels(shape, op):
    """Last-axis sums of rows of >= 1024 floats (four rows per warp once there
    are enough lanes, read as 128-byte segments when a row is whole segments,
    the staged kernel below that): ragged last tiles, a tail
    of len % 8 elements, lanes not a multiple of four or of the 32 rows per
    block, NaN and -0.0 in the data."""
    x = O.normal(int(np.prod(shape)), 62, 0, 2).reshape(shape)
    flat = x.reshape(-1, shape[-1])
    flat[0, 3] = np.nan
    flat[-1, :] = -0.0
    got = getattr(rt, f"{op}_dim")(dev(x), len(shape) - 1).to_numpy()
    assert_bits_equal(got, O.reduce_dim(op, x, len(shape) - 1), f"{op}_dim {shape}")


@pytest.mark.parametrize("shape,dim", [((4936, 1), 0), ((1512, 36, 57, 1), 2), ((83, 14, 1), 1),
                                       ((6, 5515, 16, 1), 2), ((13605, 1, 22, 1), 2),
                                       ((1 << 20, 1), 0), ((3, 1 << 19, 1, 1), 1),
                                       ((40, 70000, 1), 1), ((5, 1), 0), ((7, 3, 1, 1), 0),
                                       ((4, 1 << 18, 1), 1), ((5, 1 << 18, 1), 1)])
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_dim_reduction_before_trailing_unit_axes(shape, dim, op):
    """A non-last axis followed only by length-1 axes: the lanes are
    contiguous, but ndarray's minimum-stride axis is still the last one, so
    sum_axis adds each lane as one row-order chain from 0.0 (not the
    eight-chain lane fold).  The long single lanes take the ordered-sum
    kernels."""
    x = O.normal(int(np.prod(shape)), 63, 0, 2).reshape(shape)
    x.reshape(-1)[1] = -0.0
    got = getattr(rt, f"{op}_dim")(dev(x), dim).to_numpy()
    assert_bits_equal(got, O.reduce_dim(op, x, dim), f"{op}_dim {shape} dim={dim}")


@pytest.mark.parametrize("shape,dim", [((1512, 36, 57, 1), 2), ((4936, 1), 0), ((59, 96, 1), 1),
                                       ((50000, 1), 0), ((4, 3000, 1), 1), ((3, 1 << 19, 1), 1),
                                       ((65537, 2048, 1), 1)])
def test_softmax_before_trailing_unit_axes(shape, dim):
    # (65537, 2048, 1): the four-pass row path runs its rows in launches of
    # 65535; the last one holds two rows
    x = (O.normal(int(np.prod(shape)), 64, 0, 3)).reshape(shape)
    got = rt.softmax(dev(x), dim).to_numpy()
    assert_bits_equal(got, O.softmax(x, dim), f"softmax {shape} dim={dim}")


def test_max_dim_with_nan_and_zero_lanes():
    x = O.normal(6 * 40, 47).reshape(6, 40)
    x[0, 10] = np.nan
    x[1, 39] = np.nan
    x[2, :] = -np.abs(x[2, :])
    x[2, 5], x[2, 20] = 0.0, -0.0
    x[3, :] = np.nan
    for dim in (0, 1):
        assert_bits_equal(rt.max_dim(dev(x), dim).to_numpy(), O.reduce_dim("max", x, dim))


# ---------------------------------------------------------------- cfg 5
ADAMW = dict(lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, t=10)


def _adamw_inputs(n, offset=0):
    p = O.normal(n, 51, 0.0, 0.02, offset)
    g = O.normal(n, 52, 0.0, 1e-2, offset)
    m = O.normal(n, 53, 0.0, 1e-3, offset)
    v = O.uniform(n, 54, 0.0, 1e-4, offset)
    return p, g, m, v


def test_cfg5_adamw_full_size_chunked():
    n = 1 << 30
    chunk = 1 << 26
    lib = N.lib()
    ts = [rt.Tensor([n]) for _ in range(4)]
    for off in range(0, n, chunk):
        for t, arr in zip(ts, _adamw_inputs(chunk, off)):
            N.check(lib.rtc_memcpy_h2d(0, ctypes.c_void_p(t.ptr + 4 * off),
                                       arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes))
    p, g, m, v = ts
    # in place, as an optimizer step uses it
    N.check(lib.rtc_adamw_update(p.desc, g.desc, m.desc, v.desc, ADAMW["lr"], ADAMW["b1"],
                                 ADAMW["b2"], ADAMW["eps"], ADAMW["wd"], ADAMW["t"],
                                 p.desc, m.desc, v.desc))
    rt.synchronize()
    out = np.empty(chunk, dtype=np.float32)
    for off in range(0, n, chunk):
        hp, hg, hm, hv = _adamw_inputs(chunk, off)
        rc, wp, wm, wv = O.adamw(hp, hg, hm, hv, ADAMW["lr"], ADAMW["b1"], ADAMW["b2"],
                                 ADAMW["eps"], ADAMW["wd"], ADAMW["t"])
        assert rc == 0
        for t, want, name in ((p, wp, "p"), (m, wm, "m"), (v, wv, "v")):
            N.check(lib.rtc_memcpy_d2h(0, out.ctypes.data_as(ctypes.c_void_p),
                                       ctypes.c_void_p(t.ptr + 4 * off), out.nbytes))
            assert_bits_equal(out, want, f"adamw {name} @ {off}")


@pytest.mark.parametrize("n", [1, 7, 1 << 20, (1 << 20) + 3])
def test_adam_and_adamw_small(n):
    p, g, m, v = _adamw_inputs(n)
    for wd in (0.0, 0.01):
        po, mo, vo = rt.adamw_update(dev(p), dev(g), dev(m), dev(v), 1e-3, 0.9, 0.999, 1e-8, wd, 3)
        _, wp, wm, wv = O.adamw(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, wd, 3)
        assert_bits_equal(po.to_numpy(), wp, "p")
        assert_bits_equal(mo.to_numpy(), wm, "m")
        assert_bits_equal(vo.to_numpy(), wv, "v")
    po, mo, vo = rt.adam_update(dev(p), dev(g), dev(m), dev(v), 1e-3, 0.9, 0.999, 1e-8, 1)
    _, wp, wm, wv = O.adam(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 1)
    assert_bits_equal(po.to_numpy(), wp, "adam p")


def test_sgd_rules():
    n = 10007
    p, g, vel = O.normal(n, 61), O.normal(n, 62), O.normal(n, 63)
    want = np.empty_like(p)
    O.lib().rto_sgd_update(O.p(p), O.p(g), n, 0.1, O.p(want))
    assert_bits_equal(rt.sgd_update(dev(p), dev(g), 0.1).to_numpy(), want, "sgd")
    wp, wv = np.empty_like(p), np.empty_like(p)
    O.lib().rto_sgd_momentum_update(O.p(p), O.p(g), O.p(vel), n, 0.1, 0.9, O.p(wp), O.p(wv))
    po, vo = rt.sgd_momentum_update(dev(p), dev(g), dev(vel), 0.1, 0.9)
    assert_bits_equal(po.to_numpy(), wp, "sgd momentum p")
    assert_bits_equal(vo.to_numpy(), wv, "sgd momentum v")


# ---------------------------------------------------------------- misc
def test_device_generator_matches_host_generator():
    n = (1 << 20) + 5
    t = rt.Tensor([n])
    N.check(N.lib().rtc_fill_uniform(t.desc, 77, 1000, -1.0, 1.0))
    assert_bits_equal(t.to_numpy(), O.uniform(n, 77, -1.0, 1.0, offset=1000), "uniform")
    N.check(N.lib().rtc_fill_normal(t.desc, 78, 0, 0.0, 2.0))
    np.testing.assert_allclose(t.to_numpy(), O.normal(n, 78, 0.0, 2.0), rtol=1e-6, atol=1e-6)


def test_errors_raise_valueerror_on_gpu_too():
    a, b = dev(np.ones(4, np.float32)), dev(np.ones(5, np.float32))
    with pytest.raises(ValueError, match="Shape mismatch in element-wise addition"):
        rt.add(a, b)


# ---------------------------------------------------------------- shards
def test_device_shard_summaries_match_and_combine():
    from rusttorch_b200 import sharded
    from tests.test_sharded_gloo import CASES, _split, summary_of

    for name, make in CASES.items():
        x = make()
        parts = []
        for shard in _split(x, 2, name):
            shard = np.ascontiguousarray(shard)
            d = dev(shard)
            s = sharded.ShardSummary()
            sharded._bind(N.lib())
            N.check(N.lib().rtc_shard_summary_local(d.desc, ctypes.byref(s)))
            w = summary_of(shard)
            assert s.count == w.count and s.max_kind == w.max_kind and s.first_nan == w.first_nan
            for fld in ("max", "min_nonnan"):
                a, b = np.float32(getattr(s, fld)), np.float32(getattr(w, fld))
                assert (np.isnan(a) and np.isnan(b)) or a.view(np.uint32) == b.view(np.uint32), \
                    (name, fld, a, b)
            parts.append(s)
        tot, mean, mx, mn = sharded.combine(parts)
        for got, op in ((mx, "max"), (mn, "min")):
            want = O.scalar_reduce(op, x)[1]
            assert (np.isnan(got) and np.isnan(want)) or \
                np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), (name, op)


def test_bounded_wait_timeout_is_reported_and_context_survives():
    """The failure path of the TMA rings' bounded waits, made to run out on
    purpose: a one-thread kernel waits 50 ms on an mbarrier nothing arrives
    on, raises the device flag and returns; rtc_synchronize reports it once,
    and the GPU keeps working (no fault, no hang)."""
    import ctypes
    L = N.lib()
    N.check(L.rtc_synchronize())
    N.check(L.rtc_selftest_bounded_wait())
    r = L.rtc_synchronize()
    assert not r.success and r.code == N.BACKEND_ERROR
    msg = ctypes.string_at(r.error_msg).decode()
    L.rtc_free_error_message(r.error_msg)
    assert "gave up waiting" in msg
    N.check(L.rtc_synchronize())                      # the flag was cleared
    x = O.normal(1 << 20, 61)
    assert_bits_equal(rt.relu(dev(x)).to_numpy(), O.unary("relu", x), "relu after the probe")


def test_concurrent_host_threads():
    """Four host threads issuing ops at once (each on its own per-thread
    stream, ctypes releasing the GIL): every result matches the oracle."""
    import threading
    errors = []

    def work(k):
        try:
            x = O.normal(256 * 1024, 70 + k).reshape(256, 1024)
            y = O.normal(256 * 1024, 80 + k).reshape(256, 1024)
            for _ in range(5):
                dx, dy = dev(x), dev(y)
                assert_bits_equal(rt.softmax(dx, 1).to_numpy(), O.softmax(x, 1), f"t{k} softmax")
                assert_bits_equal(rt.add(dx, dy).to_numpy(), O.binary("add", x, y), f"t{k} add")
                assert_bits_equal(rt.sum_dim(dx, 0).to_numpy(), O.reduce_dim("sum", x, 0),
                                  f"t{k} sum_dim")
                _check_sum(rt.sum(dx), x)
        except Exception as e:          # collected and re-raised below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(k,)) for k in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
