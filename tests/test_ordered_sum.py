"""The losses' ordered f32 sums (ndarray's eight-chain unrolled_fold and
Iterator::sum's one chain), computed on the GPU in parallel from per-binade
integer translations (rusttorch_b200/csrc/rt_osum.cuh, ordered_sum.cu).

Every case compares the f32 result bit for bit with the oracle's sequential
fold (oracle/rt_oracle.c rto_unrolled_sum_f32 / rto_chain_sum_f32).  The
inputs aim at the algorithm's edges: rounding ties (x/ulp an odd multiple of
1/2, where the move depends on the running sum's parity), sums that cross
binades up and down, zero runs with both signs of zero, NaN/inf, overflow,
subnormal terms, ragged lengths and the full loss sizes.
"""
import ctypes

import numpy as np
import pytest

from tests import _oracle as O

F = np.float32


def _rng(seed):
    return np.random.default_rng(seed)


def _cases():
    r = _rng(7)
    n20 = 1 << 20
    idx = np.arange(n20)
    out = {
        "uniform": r.random(n20, dtype=F),
        "squares_of_normal": (r.standard_normal(n20 + 13).astype(F) ** 2).astype(F),
        "ragged_1000003": r.random(1000003, dtype=F),
        "ties_k_2^-24_from_1": np.where(idx == 0, F(1), (r.integers(0, 4, n20) * 2.0 ** -24)).astype(F),
        "ties_odd_halves": np.where(idx[: 1 << 19] < 8, F(1.5),
                                    (1 + 2 * r.integers(0, 3, 1 << 19)) * 2.0 ** -25).astype(F),
        "ties_big_sum": np.where(idx < 8, F(3.0e6), 0.5 + r.integers(0, 3, n20)).astype(F),
        "normal_mixed_sign": r.standard_normal(n20).astype(F),
        "up_then_down": np.where(idx < n20 // 2, r.random(n20, dtype=F), -r.random(n20, dtype=F)),
        "all_pos_zero": np.zeros(1 << 18, F),
        "all_neg_zero": np.full(1 << 18, -0.0, F),
        "neg_zero_then_pos_zero": np.where(np.arange(1 << 18) == 100000, F(0), F(-0.0)).astype(F),
        "zeros_then_values": np.where(idx < 300000, F(0), r.random(n20, dtype=F)).astype(F),
        "zero_blocks_inside": np.where((idx // 4096) % 3 == 0, F(0), r.random(n20, dtype=F)),
        "overflow_to_inf": (F(3.0e33) * r.random(1 << 18, dtype=F)).astype(F),
        "subnormal_terms": (F(1e-40) * r.random(1 << 18, dtype=F)).astype(F),
        "tiny_terms": (F(1e-30) * r.random(n20, dtype=F)).astype(F),
        "huge_then_small": np.where(idx < 8, F(1e30), r.random(n20, dtype=F)).astype(F),
        "ones": np.ones(n20, F),
        "cancel_to_zero": np.where(np.arange(1 << 18) & 1, F(-1), F(1)).astype(F),
        "geometric_growth": (np.ldexp(F(1), (np.arange(1 << 18) // 2048).astype(np.int32) - 60)
                             * (1 + r.random(1 << 18, dtype=F))).astype(F),
        "negative_uniform": -r.random(n20, dtype=F),
        "n5": r.random(5, dtype=F),
        "n300": r.random(300, dtype=F),
        "n4100": r.random(4100, dtype=F),
    }
    nan = r.random(1 << 18, dtype=F)
    nan[77777] = np.nan
    out["one_nan"] = nan
    inf = r.random(1 << 18, dtype=F)
    inf[77777] = np.inf
    out["one_inf"] = inf
    both = r.random(1 << 18, dtype=F)
    both[7777], both[200000] = np.inf, -np.inf
    out["inf_then_neg_inf"] = both
    # a sum that turns infinite early in a long chain: the walk skips to the
    # blocks that can still change it (here a NaN, and an opposite infinity)
    long_inf = r.random((1 << 22) + 9, dtype=F)
    long_inf[10] = np.inf
    out["inf_early_long"] = long_inf.copy()
    long_inf[3_000_001] = np.nan
    out["inf_early_then_nan_long"] = long_inf.copy()
    long_inf[3_000_001] = -np.inf
    out["inf_early_then_neg_inf_long"] = long_inf
    return out


CASES = _cases()


def _gpu_sum(x, chains, init=-0.0):
    import rusttorch_b200 as rt
    from rusttorch_b200 import _native as N
    v = ctypes.c_float()
    t = rt.Tensor.from_numpy(np.ascontiguousarray(x, F))
    N.check(N.lib().rtc_selftest_ordered_sum(t.desc, chains, init, ctypes.byref(v)))
    return F(v.value)


def _same(a, b):
    a, b = F(a), F(b)
    return (np.isnan(a) and np.isnan(b)) or a.view(np.uint32) == b.view(np.uint32)


def test_oracle_ordered_sums_restate_the_folds():
    # CPU: the oracle's two folds against a Python loop of f32 adds
    x = _rng(3).random(1003, dtype=F)
    p = [F(0)] * 8
    for i in range(1000):
        p[i % 8] = F(p[i % 8] + x[i])
    acc = F(0)
    for j in range(4):
        acc = F(acc + F(p[j] + p[j + 4]))
    for v in x[1000:]:
        acc = F(acc + v)
    assert _same(O.unrolled_sum_f32(x), acc)
    s = F(-0.0)
    for v in x:
        s = F(s + v)
    assert _same(O.chain_sum_f32(x), s)
    assert O.chain_sum_f32(np.full(4, -0.0, F)).view(np.uint32) == 0x80000000


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_gpu_ordered_sum_eight_chains(name):
    x = CASES[name]
    want = O.unrolled_sum_f32(x)
    got = _gpu_sum(x, 8)
    assert _same(got, want), (name, got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_gpu_ordered_sum_one_chain(name):
    x = CASES[name]
    want = O.chain_sum_f32(x, -0.0)
    got = _gpu_sum(x, 1, -0.0)
    assert _same(got, want), (name, got, want)


@pytest.mark.gpu
def test_gpu_ordered_sum_one_chain_init_and_empty():
    x = np.full(1000, -0.0, F)
    assert _gpu_sum(x, 1, -0.0).view(np.uint32) == 0x80000000
    assert _gpu_sum(x, 1, 0.0).view(np.uint32) == 0
    assert _gpu_sum(x, 8).view(np.uint32) == 0          # ndarray's chains start at +0
    y = _rng(5).random(777, dtype=F)
    assert _same(_gpu_sum(y, 1, 3.5), O.chain_sum_f32(y, 3.5))
    assert _same(_gpu_sum(np.zeros(0, F), 1, -0.0), F(-0.0))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(6))
def test_gpu_ordered_sum_random_lengths(seed):
    r = _rng(100 + seed)
    n = int(r.integers(1, 3_000_000))
    scale = F(10.0) ** r.integers(-20, 20)
    x = (r.random(n, dtype=F) * scale).astype(F)
    if seed % 2:
        x = (x * np.where(r.random(n) < 0.1, F(-1), F(1))).astype(F)
    assert _same(_gpu_sum(x, 8), O.unrolled_sum_f32(x)), n
    assert _same(_gpu_sum(x, 1), O.chain_sum_f32(x)), n


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["mse", "l1", "smooth_l1", "bce", "ce"])
def test_gpu_losses_full_size(kind):
    # cfg1's 2^24 elements through the loss entry points
    import math

    import rusttorch_b200 as rt
    n = 1 << 24
    if kind in ("bce", "ce"):
        p = O.uniform(n, 31, 0.0, 1.0)
        t = (O.uniform(n, 32, 0.0, 1.0) > 0.5).astype(F)
        par = (1e-7,)
    else:
        p, t = O.normal(n, 31), O.normal(n, 32)
        par = (0.75,) if kind == "smooth_l1" else ()
    api = {"mse": rt.mse_loss, "l1": rt.l1_loss, "smooth_l1": rt.smooth_l1_loss,
           "bce": rt.binary_cross_entropy_loss, "ce": rt.cross_entropy_loss}[kind]
    got = api(rt.Tensor.from_numpy(p), rt.Tensor.from_numpy(t), *par)
    want = O.loss(kind, p, t, *par)
    if kind in ("bce", "ce"):
        assert math.isclose(got, want, rel_tol=1e-6), (got, want)
    else:
        assert got == want, (got, want)
