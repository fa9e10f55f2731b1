"""Single-process sharded ops (rtc_sharded_*) against the oracle.

A tensor is cut into shards spread round-robin over every visible GPU (all
on GPU 0 on a one-GPU box), the sharded entry point runs them all, and the
concatenated result must equal the oracle's result for the whole tensor,
bit for bit (softmax in the tolerance math mode: within 1e-6 relative
error or 4 ulp, as on one GPU).
"""
import numpy as np
import pytest

import rusttorch_b200 as rt
from rusttorch_b200 import _native as N
from tests import _oracle as O
from tests.test_tolerance_gpu import assert_bits_equal, assert_within_tolerance

pytestmark = pytest.mark.gpu


def ngpu():
    import torch
    return max(1, torch.cuda.device_count())


def shards_of(x, cuts, axis=0):
    parts = np.split(x, cuts, axis=axis)
    return [rt.Tensor.from_numpy(np.ascontiguousarray(p), device=i % ngpu())
            for i, p in enumerate(parts)]


def test_sharded_add_mul_scalar():
    n = (1 << 22) + 5
    a, b = O.uniform(n, 1), O.uniform(n, 101)
    cuts = [1, 1_000_003, 2_500_000, 4_000_000]
    out = rt.sharded_add_mul_scalar(shards_of(a, cuts), shards_of(b, cuts), 0.5)
    got = np.concatenate([t.to_numpy() for t in out])
    assert_bits_equal(got, O.scalar_op("mul_scalar", O.binary("add", a, b), 0.5), "add->mul")


def test_sharded_softmax_row_blocks():
    x = O.normal(4096 * 4096, 4, 0.0, 2.0).reshape(4096, 4096)
    cuts = [1000, 1001, 3000]
    out = rt.sharded_softmax(shards_of(x, cuts), 1)
    got = np.concatenate([t.to_numpy() for t in out])
    assert_within_tolerance(got, O.softmax(x, 1), "sharded softmax")
    with rt.math_mode("exact"):
        out = rt.sharded_softmax(shards_of(x, cuts), 1)
        assert_bits_equal(np.concatenate([t.to_numpy() for t in out]), O.softmax(x, 1),
                          "sharded softmax (exact)")


@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_sharded_dim0_column_blocks(op):
    """cfg3's dim-0 reduction split into column blocks: each block is its
    own contiguous [R, C_i] tensor, reduced on its GPU."""
    x = O.uniform(2048 * 4096, 3).reshape(2048, 4096)
    cuts = [1024, 1027, 3000]
    out = getattr(rt, f"sharded_{op}_dim")(shards_of(x, cuts, axis=1), 0)
    got = np.concatenate([t.to_numpy() for t in out])
    assert_bits_equal(got, O.reduce_dim(op, x, 0), f"sharded {op}_dim(0)")


@pytest.mark.parametrize("op", ["sum", "max"])
def test_sharded_dim1_row_blocks(op):
    x = O.uniform(2048 * 4096, 3).reshape(2048, 4096)
    out = getattr(rt, f"sharded_{op}_dim")(shards_of(x, [700, 1500]), 1)
    got = np.concatenate([t.to_numpy() for t in out])
    assert_bits_equal(got, O.reduce_dim(op, x, 1), f"sharded {op}_dim(1)")


def test_sharded_adamw_in_place():
    n = (1 << 22) + 3
    p, g = O.normal(n, 51, 0, 0.02), O.normal(n, 52, 0, 1e-2)
    m, v = O.normal(n, 53, 0, 1e-3), O.uniform(n, 54, 0.0, 1e-4)
    cuts = [1, 2_000_000, 3_000_001]
    P, G, M, V = (shards_of(t, cuts) for t in (p, g, m, v))
    rt.sharded_adamw_update(P, G, M, V, 1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
    rc, wp, wm, wv = O.adamw(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
    assert rc == 0
    for name, shards, want in (("p", P, wp), ("m", M, wm), ("v", V, wv)):
        assert_bits_equal(np.concatenate([t.to_numpy() for t in shards]), want, f"adamw {name}")


def test_sharded_errors_launch_nothing():
    """A bad shard (or bad hyperparameter) is reported before any shard is
    touched."""
    x = O.normal(1000, 5)
    P = shards_of(x, [500])
    G = shards_of(x, [500])
    M = shards_of(x, [500])
    V = [rt.Tensor.from_numpy(np.zeros(500, np.float32), device=0),
         rt.Tensor.from_numpy(np.zeros(7, np.float32), device=1 % ngpu())]
    with pytest.raises(N.RusttorchError) as e:
        rt.sharded_adamw_update(P, G, M, V, 1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
    assert e.value.code == N.SHAPE_MISMATCH
    assert_bits_equal(P[0].to_numpy(), x[:500], "untouched after a shape error")
    V = shards_of(np.abs(x), [500])
    with pytest.raises(N.RusttorchError) as e:
        rt.sharded_adamw_update(P, G, M, V, -1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
    assert e.value.code == N.INVALID_ARGUMENT
    assert_bits_equal(P[1].to_numpy(), x[500:], "untouched after a hyperparameter error")
    with pytest.raises(N.RusttorchError) as e:
        rt.sharded_softmax(shards_of(x.reshape(100, 10), [50]), 0)
    assert e.value.code == N.INVALID_ARGUMENT
