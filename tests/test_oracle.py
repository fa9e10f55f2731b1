"""Pin the CPU oracle (oracle/rt_oracle.c) before it is trusted as the checker.

1. The reference's own known-answer tests for this path
   (rusttorch-core/src/ops/reduction.rs:157-247, simd.rs:408-415,
   activation.rs:417-490, optimizer.rs:527-563), restated here.
2. Analytic known answers (sigmoid(0) = 0.5, softmax rows sum to 1, ...).
3. tests/golden/golden.npz, produced by an independent pure-Python/numpy
   restatement (tests/golden/make_golden.py): bit-exact where the op is plain
   IEEE arithmetic or a reduction, within a few ulp where Python's math (not
   glibc) supplied a transcendental.
"""
from pathlib import Path

import numpy as np
import pytest

from tests import _oracle as O

RTO_OK, RTO_SHAPE, RTO_DTYPE, RTO_EMPTY, RTO_DIM, RTO_ARG = range(6)
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


def f32(xs):
    return np.asarray(xs, dtype=np.float32)


def bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32)


def ulp_diff(a, b):
    """|a - b| in ulps of float32 (NaN == NaN counts as equal)."""
    ia = bits(a).astype(np.int64)
    ib = bits(b).astype(np.int64)
    ia = np.where(ia < 0x80000000, ia, 0x80000000 - ia)
    ib = np.where(ib < 0x80000000, ib, 0x80000000 - ib)
    d = np.abs(ia - ib)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.where(both_nan, 0, d)


# ---- 1. the reference's known-answer tests -------------------------------
def test_sum_kat():                       # reduction.rs:157-161
    assert O.sum(f32([1, 2, 3, 4])) == 10.0


def test_mean_kat():                      # reduction.rs:164-168
    assert O.scalar_reduce("mean", f32([1, 2, 3, 4])) == (RTO_OK, 2.5)


def test_max_kat():                       # reduction.rs:171-175
    assert O.scalar_reduce("max", f32([1, 5, 3, 2])) == (RTO_OK, 5.0)


def test_min_kat():                       # reduction.rs:178-182
    assert O.scalar_reduce("min", f32([3, 1, 5, 2])) == (RTO_OK, 1.0)


def test_sum_empty_is_zero():             # reduction.rs:210-214
    assert O.sum(f32([])) == 0.0


@pytest.mark.parametrize("op", ["mean", "max", "min"])
def test_empty_reductions_error(op):      # reduction.rs:198-236
    assert O.scalar_reduce(op, f32([]))[0] == RTO_EMPTY


def test_sum_dim_shapes():                # reduction.rs:185-195
    assert O.reduce_dim("sum", f32([1, 2, 3, 4, 5, 6]).reshape(2, 3), 0).shape == (3,)
    assert O.reduce_dim("mean", f32([2, 4, 6, 8]).reshape(2, 2), 1).shape == (2,)


def test_dim_out_of_range():              # reduction.rs:239-247, activation.rs:428-437
    x = np.ones((2, 2), dtype=np.float32)
    with pytest.raises(ValueError, match="rc=4"):
        O.reduce_dim("sum", x, 5)
    with pytest.raises(ValueError, match="rc=4"):
        O.softmax(np.ones((2, 3), dtype=np.float32), 5)


def test_elu_negative_alpha():            # activation.rs:481-490
    with pytest.raises(ValueError):
        O.unary("elu", f32([1.0]), -0.5)


def test_fma_kat():                       # simd.rs:408-415: [3, 7, 13]
    np.testing.assert_array_equal(O.fma(f32([1, 2, 3]), f32([2, 3, 4]), f32([1, 1, 1])),
                                  f32([3, 7, 13]))


def test_adam_zero_timestep():            # optimizer.rs:548-562
    one = f32([1.0])
    assert O.adam(one, f32([0.1]), f32([0]), f32([0]), 0.001, 0.9, 0.999, 1e-8, 0)[0] == RTO_ARG


def test_adamw_negative_decay():          # optimizer.rs:392-397
    one = f32([1.0])
    assert O.adamw(one, one, one, one, 0.001, 0.9, 0.999, 1e-8, -0.01, 1)[0] == RTO_ARG


def test_sgd_negative_lr():               # optimizer.rs:533-545
    p = f32([1.0])
    out = np.empty_like(p)
    assert O.lib().rto_sgd_update(O.p(p), O.p(f32([0.1])), 1, -0.1, O.p(out)) == RTO_ARG


# ---- 2. analytic known answers ----------------------------------------------
def test_sigmoid_of_zero():
    assert O.unary("sigmoid", f32([0.0]))[0] == 0.5


def test_relu_signed():
    r = O.unary("relu", f32([-2, -1, -0.0, 0, 1, 2, np.nan]))
    np.testing.assert_array_equal(bits(r), bits(f32([0, 0, 0, 0, 1, 2, 0])))


def test_leaky_relu_signed():
    r = O.unary("leaky_relu", f32([-2.0, 3.0]), 0.01)
    np.testing.assert_array_equal(r, f32([np.float32(-2.0) * np.float32(0.01), 3.0]))


def test_elu_selu_at_zero():
    assert O.unary("elu", f32([0.0]), 1.0)[0] == 0.0
    assert O.unary("selu", f32([0.0]))[0] == 0.0


def test_softmax_rows_sum_to_one():
    x = O.normal(6 * 50, 7, 0.0, 2.0).reshape(6, 50)
    for dim in (0, 1):
        s = O.softmax(x, dim).astype(np.float64).sum(axis=dim)
        np.testing.assert_allclose(s, 1.0, rtol=1e-5)


def test_adam_first_step_closed_form():
    # t = 1: m_hat = g, v_hat = g^2, so p' = p - lr * g / (|g| + eps).
    p, g = f32([1.0, -2.0, 0.5]), f32([0.1, -0.2, 0.3])
    z = np.zeros(3, dtype=np.float32)
    rc, po, mo, vo = O.adam(p, g, z, z, 0.001, 0.9, 0.999, 1e-8, 1)
    assert rc == RTO_OK
    expect = p.astype(np.float64) - 0.001 * np.sign(g)
    np.testing.assert_allclose(po, expect, rtol=0, atol=1e-6)
    np.testing.assert_allclose(mo, 0.1 * g, rtol=1e-6)
    # (1 - beta2) is formed in f32 from f32(0.999) (optimizer.rs:300)
    one_minus_b2 = float(np.float32(1.0) - np.float32(0.999))
    np.testing.assert_allclose(vo, one_minus_b2 * g.astype(np.float64) ** 2, rtol=1e-6)


def test_max_min_fold_semantics():
    # Equal keeps the later element for max and the earlier for min; NaN
    # compares Equal (the max fold restarts after it, the min fold skips it
    # unless it comes first).
    nan = np.nan
    cases = [
        (f32([0.0, -0.0]), -0.0, 0.0),
        (f32([-0.0, 0.0]), 0.0, -0.0),
        (f32([1, nan, 0.5]), 0.5, 0.5),
        (f32([3, 1, nan]), nan, 1.0),
        (f32([nan, 1, 2]), 2.0, nan),
    ]
    for x, mx, mn in cases:
        _, got_mx = O.scalar_reduce("max", x)
        _, got_mn = O.scalar_reduce("min", x)
        assert (np.isnan(mx) and np.isnan(got_mx)) or bits(got_mx) == bits(mx), (x, got_mx)
        assert (np.isnan(mn) and np.isnan(got_mn)) or bits(got_mn) == bits(mn), (x, got_mn)


# ---- 3. golden fixtures (independent restatement) ---------------------------
EXACT_BINARY = ["add", "sub", "mul"]


@pytest.mark.parametrize("op", EXACT_BINARY)
def test_golden_binary(op):
    np.testing.assert_array_equal(bits(O.binary(op, GOLD["a"], GOLD["b"])), bits(GOLD[op]))


def test_golden_div():
    np.testing.assert_array_equal(bits(O.binary("div", GOLD["a"], GOLD["b_nz"])),
                                  bits(GOLD["div"]))


def test_golden_scalar_and_fma():
    a, b, c = GOLD["a"], GOLD["b"], GOLD["c"]
    np.testing.assert_array_equal(bits(O.scalar_op("add_scalar", a, 10.0)), bits(GOLD["add_scalar"]))
    np.testing.assert_array_equal(bits(O.scalar_op("mul_scalar", a, 0.5)), bits(GOLD["mul_scalar"]))
    np.testing.assert_array_equal(bits(O.scalar_op("mul_scalar", O.binary("add", a, b), 0.5)),
                                  bits(GOLD["add_mul_scalar"]))
    np.testing.assert_array_equal(bits(O.fma(a, b, c)), bits(GOLD["fma"]))


def test_golden_relu_family():
    a = GOLD["a"]
    np.testing.assert_array_equal(bits(O.unary("relu", a)), bits(GOLD["relu"]))
    np.testing.assert_array_equal(bits(O.unary("leaky_relu", a, 0.01)), bits(GOLD["leaky_relu"]))
    np.testing.assert_array_equal(bits(O.unary("softsign", a)), bits(GOLD["softsign"]))


# Python's math rounds to nearest double; glibc's f32 functions are within 1
# ulp of the correctly rounded result, and the ops below add at most a couple
# of roundings on top.  Inputs where the op cancels catastrophically (GELU's
# 1 + tanh for large negative x) are excluded from the ulp check.
@pytest.mark.parametrize("op,max_ulp", [("sigmoid", 2), ("swish", 2), ("tanh", 2), ("elu", 2),
                                        ("selu", 3), ("softplus", 2), ("mish", 4), ("gelu", 4)])
def test_golden_transcendental(op, max_ulp):
    a = GOLD["a"]
    got = O.unary(op, a, 1.0) if op == "elu" else O.unary(op, a)
    want = GOLD[op]
    mask = np.ones(a.size, dtype=bool)
    if op == "gelu":
        mask = a > -3.0
    if op in ("elu", "selu"):
        mask = (a > 0) | (a < -0.05)       # exp(x) - 1 cancels near 0-
    d = ulp_diff(got[mask], want[mask]).astype(np.float64)
    allowed = np.full(d.shape, float(max_ulp))
    if op == "gelu":
        # (0.5x)(1 + t) amplifies a 1-ulp difference in t = tanh(z) by |t|/|1+t|.
        import math
        k = float(np.float32(math.sqrt(float(np.float32(2.0) / np.float32(math.pi)))))
        x = a[mask].astype(np.float64)
        t = np.tanh(k * (x + 0.044715 * x ** 3))
        allowed += 2.0 * np.abs(t) / np.maximum(np.abs(1.0 + t), 1e-30)
    bad = d > allowed
    assert not bad.any(), (op, a[mask][bad][:3], got[mask][bad][:3], want[mask][bad][:3])


def test_golden_reductions():
    a = GOLD["a"]
    assert O.sum(a) == GOLD["sum"][0]
    assert O.scalar_reduce("mean", a)[1] == GOLD["mean"][0]
    assert O.scalar_reduce("max", a)[1] == GOLD["max"][0]
    assert O.scalar_reduce("min", a)[1] == GOLD["min"][0]
    m2 = GOLD["m2"]
    for op in ("sum", "mean", "max"):
        for dim in (0, 1):
            np.testing.assert_array_equal(bits(O.reduce_dim(op, m2, dim)),
                                          bits(GOLD[f"{op}_dim{dim}"]), err_msg=f"{op}_dim{dim}")


def test_oracle_sum_axis_order_before_trailing_unit_axes():
    # ndarray 0.15 sum_axis folds lanes with unrolled_fold only along the
    # minimum-stride axis: min_by_key over the axes in reverse keeps the LAST
    # axis of equal |stride|, and a length-1 axis after `dim` has stride 1 in
    # the default strides, so [n, 1] summed over dim 0 is the row-order chain
    # 0 + x0 + x1 + ..., not the eight-chain lane fold.
    x = O.normal(4099, 65, 0, 3)
    chain = np.float32(0.0)
    for v in x:
        chain = np.float32(chain + v)
    lane = O.unrolled_sum_f32(x)
    assert bits(chain) != bits(lane)          # the two orders differ on this input
    for shape, dim in (((4099, 1), 0), ((1, 4099, 1, 1), 1)):
        got = O.reduce_dim("sum", x.reshape(shape), dim).ravel()[0]
        assert bits(got) == bits(chain), shape
    assert bits(O.reduce_dim("sum", x.reshape(1, 4099), 1)[0]) == bits(lane)
    s = O.softmax(x.reshape(4099, 1), 0).ravel()
    e = np.exp(x.astype(np.float64) - x.max()).astype(np.float32)
    assert abs(float(s.sum()) - 1.0) < 1e-4 and np.allclose(s, e / e.sum(), rtol=1e-5)


def test_golden_softmax():
    d = ulp_diff(O.softmax(GOLD["m2"], 1), GOLD["softmax_dim1"])
    assert d.max() <= 4


def test_golden_adamw():
    rc, po, mo, vo = O.adamw(GOLD["adam_p"], GOLD["adam_g"], GOLD["adam_m"], GOLD["adam_v"],
                             1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
    assert rc == RTO_OK
    np.testing.assert_array_equal(bits(po), bits(GOLD["adamw_p_out"]))
    np.testing.assert_array_equal(bits(mo), bits(GOLD["adamw_m_out"]))
    np.testing.assert_array_equal(bits(vo), bits(GOLD["adamw_v_out"]))


def test_generator_is_counter_based():
    full = O.uniform(1000, 42)
    part = O.uniform(100, 42, offset=500)
    np.testing.assert_array_equal(full[500:600], part)
    assert full.min() >= -1.0 and full.max() < 1.0
    z = O.normal(200000, 3, 0.0, 2.0)
    assert abs(float(z.mean())) < 0.03 and abs(float(z.std()) - 2.0) < 0.03
