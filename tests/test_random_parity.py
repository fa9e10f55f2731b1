"""Seeded random sweep of shapes, axes and value mixes through the C ABI,
compared with the oracle (bit for bit, NaN equal to NaN; bce/ce within the
1e-6 relative tolerance of tests/test_losses.py).

Each case draws its own shape (1 to 4 axes, lengths log-uniform up to 70000,
so length-1 axes appear in every position), axis and values from one of nine
mixes: uniform, normal, wide exponent ranges, rounding ties (small multiples
of a power of two after a large lead term), zeros of both signs, powers of
two of mixed sign, half-integers, squares, with occasional NaN and +/-inf.
The areas are the dim reductions, softmax, broadcasting binary ops with
broadcast_add's backward fold, the losses, and the ordered f32 sums under
the losses; a last group puts inputs and outputs off the 16-byte boundary and
lets outputs alias inputs.
"""
import ctypes
import math

import numpy as np
import pytest

from tests import _oracle as O
from tests.test_parity_gpu import assert_bits_equal

# Bit-exact comparisons of the transcendental activations and softmax need
# the exact math mode (the tolerance mode is tests/test_tolerance_gpu.py).
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_math")]

F = np.float32
SEEDS = range(40)


def _values(r, n):
    kind = int(r.integers(0, 9))
    if kind == 0:
        x = r.random(n, dtype=F)
    elif kind == 1:
        x = r.standard_normal(n).astype(F)
    elif kind == 2:
        x = (r.random(n, dtype=F) * F(10.0) ** r.integers(-30, 30)).astype(F)
    elif kind == 3:
        x = (r.integers(0, 5, n) * 2.0 ** int(r.integers(-26, -20))).astype(F)
        x[: int(r.integers(0, 9))] = F(1.0 + r.integers(0, 4))
    elif kind == 4:
        x = np.where(r.random(n) < 0.5, F(0), r.random(n, dtype=F)).astype(F)
        x[r.random(n) < 0.3] = -0.0
    elif kind == 5:
        x = (r.random(n, dtype=F) - F(0.5)).astype(F)
    elif kind == 6:
        x = np.ldexp(F(1), r.integers(-40, 40, n).astype(np.int32)).astype(F) * \
            np.where(r.random(n) < 0.2, F(-1), F(1))
    elif kind == 7:
        x = (F(0.5) + r.integers(0, 3, n)).astype(F)
    else:
        x = (r.standard_normal(n) ** 2).astype(F)
    if r.random() < 0.15 and n:
        x[int(r.integers(0, n))] = [np.inf, -np.inf, np.nan][int(r.integers(0, 3))]
    if r.random() < 0.05 and n:
        x[int(r.integers(0, n))] = np.inf
        x[int(r.integers(0, n))] = -np.inf
    return x.astype(F)


def _len(r, hi):
    return int(min(hi, math.exp(r.uniform(0, math.log(hi)))))


def _shape(r, max_numel):
    nd = int(r.integers(1, 5))
    while True:
        shape = [max(1, _len(r, 70000)) for _ in range(nd)]
        if int(np.prod(shape)) <= max_numel:
            return shape


def _dev(a):
    import rusttorch_b200 as rt
    return rt.Tensor.from_numpy(np.ascontiguousarray(a, F))


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_random_dim_reductions(op, seed):
    import rusttorch_b200 as rt
    r = np.random.default_rng([1, seed, len(op)])
    shape = _shape(r, 4_000_000)
    x = _values(r, int(np.prod(shape))).reshape(shape)
    dim = int(r.integers(0, len(shape)))
    got = getattr(rt, f"{op}_dim")(_dev(x), dim).to_numpy()
    assert_bits_equal(got, O.reduce_dim(op, x, dim), f"{op}_dim {shape} dim={dim}")


@pytest.mark.parametrize("seed", SEEDS)
def test_random_softmax(seed):
    import rusttorch_b200 as rt
    r = np.random.default_rng([2, seed])
    shape = _shape(r, 2_000_000)
    x = (r.standard_normal(int(np.prod(shape))) * r.uniform(0.1, 30)).astype(F).reshape(shape)
    if r.random() < 0.2:
        x.reshape(-1)[int(r.integers(0, x.size))] = [np.inf, -np.inf, np.nan][int(r.integers(0, 3))]
    dim = int(r.integers(0, len(shape)))
    got = rt.softmax(_dev(x), dim).to_numpy()
    assert_bits_equal(got, O.softmax(x, dim), f"softmax {shape} dim={dim}")


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_random_broadcast_and_add_backward(op, seed):
    import rusttorch_b200 as rt
    r = np.random.default_rng([3, seed, len(op), ord(op[0])])
    shape = _shape(r, 2_000_000)
    sa = [d if r.random() < 0.7 else 1 for d in shape]
    sb = [d if r.random() < 0.6 else 1 for d in shape]
    if r.random() < 0.4:
        sb = sb[int(r.integers(0, len(sb))):]
    a = _values(r, int(np.prod(sa))).reshape(sa)
    b = _values(r, int(np.prod(sb))).reshape(sb)
    got = getattr(rt, f"{op}_broadcast")(_dev(a), _dev(b)).to_numpy()
    rc, want = O.broadcast(op, a, b)
    assert rc == 0
    assert_bits_equal(got, want, f"{op} {sa} {sb}")
    g = _values(r, got.size).reshape(got.shape)
    ga, gb = rt.broadcast_add_backward(_dev(g), sa, sb)
    for t, s in ((ga, sa), (gb, sb)):
        rc, w = O.reduce_to_shape(g, s)
        assert rc == 0
        assert_bits_equal(t.to_numpy(), w, f"add backward {list(got.shape)} -> {s}")


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("name", ["mse", "l1", "smooth_l1", "bce", "ce"])
def test_random_losses(name, seed):
    import rusttorch_b200 as rt
    r = np.random.default_rng([4, seed, len(name), ord(name[0])])
    n = _len(r, 2_000_000)
    if name in ("bce", "ce"):
        p = r.random(n, dtype=F)
        t = r.random(n, dtype=F) if r.random() < 0.5 else (r.random(n) < 0.5).astype(F)
        if r.random() < 0.2:
            t = (t * F(2) - F(0.5)).astype(F)      # targets outside [0, 1]
        par = (float(10.0 ** r.integers(-9, -3)),)
    else:
        p, t = _values(r, n), _values(r, n)
        par = (float(r.uniform(0.1, 3.0)),) if name == "smooth_l1" else ()
    api = {"mse": rt.mse_loss, "l1": rt.l1_loss, "smooth_l1": rt.smooth_l1_loss,
           "bce": rt.binary_cross_entropy_loss, "ce": rt.cross_entropy_loss}[name]
    got = api(_dev(p), _dev(t), *par)
    want = O.loss(name, p, t, *par)
    if math.isnan(want):
        assert math.isnan(got), (name, n, got)
    elif name in ("bce", "ce"):
        assert got == want or math.isclose(got, want, rel_tol=1e-6), (name, n, got, want)
    else:
        assert got == want, (name, n, got, want)


@pytest.mark.parametrize("seed", SEEDS)
def test_random_ordered_sums(seed):
    from rusttorch_b200 import _native as N
    r = np.random.default_rng([5, seed])
    x = _values(r, _len(r, 4_000_000))
    t = _dev(x)          # held: a descriptor does not keep its tensor's buffer alive
    for chains in (8, 1):
        init = -0.0 if chains == 8 or r.random() < 0.7 else float(F(r.standard_normal()))
        v = ctypes.c_float()
        N.check(N.lib().rtc_selftest_ordered_sum(t.desc, chains, init, ctypes.byref(v)))
        want = O.unrolled_sum_f32(x) if chains == 8 else O.chain_sum_f32(x, init)
        assert_bits_equal(np.float32(v.value), want, f"chains={chains} n={x.size}")


def _view(x, off):
    """x copied to the device `off` floats past the start of a fresh device
    buffer (whose start is 256-byte aligned: off 1-3 is not 16-byte aligned)."""
    import rusttorch_b200 as rt
    from rusttorch_b200 import _native as N
    n = x.size
    base = rt.Tensor([n + off + 1])
    h = np.zeros(n + off + 1, F)
    h[off:off + n] = x.ravel()
    N.check(N.lib().rtc_memcpy_h2d(0, ctypes.c_void_p(base.ptr), h.ctypes.data_as(ctypes.c_void_p),
                                   h.nbytes))
    return rt.Tensor.from_device_ptr(base.ptr + 4 * off, list(x.shape), owner=base)


def _out_view(shape, off):
    import rusttorch_b200 as rt
    base = rt.Tensor([int(np.prod(shape)) + off + 1])
    return rt.Tensor.from_device_ptr(base.ptr + 4 * off, list(shape), owner=base)


@pytest.mark.parametrize("seed", range(20))
def test_random_misaligned_views_and_in_place(seed):
    """Inputs and outputs off the 16-byte boundary (the kernels' vector and
    TMA paths give way to their scalar forms), outputs aliasing inputs."""
    from rusttorch_b200 import _native as N
    r = np.random.default_rng([6, seed])
    shape = _shape(r, 1_000_000)
    if r.random() < 0.3:
        shape = shape + [1]
    x = _values(r, int(np.prod(shape))).reshape(shape)
    off = int(r.integers(1, 4))
    vx = _view(x, off)
    dim = int(r.integers(0, len(shape)))
    oshape = [d for i, d in enumerate(shape) if i != dim]
    for op in ("sum", "mean", "max"):
        out = _out_view(oshape, int(r.integers(0, 4)))
        N.check(getattr(N.lib(), f"rtc_{op}_dim")(vx.desc, dim, out.desc))
        assert_bits_equal(out.to_numpy(), O.reduce_dim(op, x, dim), f"{op}_dim {shape} {dim}")
    xs = (r.standard_normal(x.size) * 3).astype(F).reshape(shape)
    vs = _view(xs, off)
    N.check(N.lib().rtc_softmax(vs.desc, dim, vs.desc))          # in place
    assert_bits_equal(vs.to_numpy(), O.softmax(xs, dim), f"softmax {shape} {dim}")
    a, b = _values(r, x.size), _values(r, x.size)
    va, vb = _view(a, off), _view(b, off)
    N.check(N.lib().rtc_div(va.desc, vb.desc, va.desc))
    assert_bits_equal(va.to_numpy(), O.binary("div", a, b), "div in place")
    N.check(N.lib().rtc_gelu(vb.desc, vb.desc))
    assert_bits_equal(vb.to_numpy(), O.unary("gelu", b), "gelu in place")
    p = _values(r, x.size)
    t = _values(r, x.size)
    import rusttorch_b200 as rt
    got = rt.mse_loss(_view(p, int(r.integers(0, 4))), _view(t, int(r.integers(0, 4))))
    want = O.loss("mse", p, t)
    assert (math.isnan(got) and math.isnan(want)) or got == want, (got, want)
