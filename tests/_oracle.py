"""ctypes access to the parity oracle (oracle/liboracle.so) for the tests.

The oracle is test infrastructure: a CPU restatement of the reference's ops
(see oracle/rt_oracle.h).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg load it.
"""
import ctypes
from ctypes import POINTER, c_double, c_float, c_int, c_size_t, c_uint64, c_void_p
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
_lib = None

F = c_void_p


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(ROOT / "oracle" / "liboracle.so"))
        sz = POINTER(c_size_t)
        sig = {
            "rto_add": (None, [F, F, F, c_size_t]), "rto_sub": (None, [F, F, F, c_size_t]),
            "rto_mul": (None, [F, F, F, c_size_t]), "rto_div": (None, [F, F, F, c_size_t]),
            "rto_add_scalar": (None, [F, c_float, F, c_size_t]),
            "rto_mul_scalar": (None, [F, c_float, F, c_size_t]),
            "rto_fused_multiply_add": (None, [F, F, F, F, c_size_t]),
            "rto_relu": (None, [F, F, c_size_t]),
            "rto_leaky_relu": (None, [F, c_float, F, c_size_t]),
            "rto_sigmoid": (None, [F, F, c_size_t]), "rto_tanh": (None, [F, F, c_size_t]),
            "rto_gelu": (None, [F, F, c_size_t]), "rto_swish": (None, [F, F, c_size_t]),
            "rto_elu": (c_int, [F, c_float, F, c_size_t]), "rto_selu": (None, [F, F, c_size_t]),
            "rto_mish": (None, [F, F, c_size_t]), "rto_softplus": (None, [F, F, c_size_t]),
            "rto_softsign": (None, [F, F, c_size_t]),
            "rto_softmax": (c_int, [F, sz, c_size_t, c_size_t, F]),
            "rto_sum": (c_double, [F, c_size_t]),
            "rto_mean": (c_int, [F, c_size_t, POINTER(c_double)]),
            "rto_max": (c_int, [F, c_size_t, POINTER(c_double)]),
            "rto_min": (c_int, [F, c_size_t, POINTER(c_double)]),
            "rto_sum_dim": (c_int, [F, sz, c_size_t, c_size_t, F]),
            "rto_mean_dim": (c_int, [F, sz, c_size_t, c_size_t, F]),
            "rto_max_dim": (c_int, [F, sz, c_size_t, c_size_t, F]),
            "rto_adam_update": (c_int, [F, F, F, F, c_size_t, c_double, c_double, c_double,
                                        c_double, c_uint64, F, F, F]),
            "rto_adamw_update": (c_int, [F, F, F, F, c_size_t, c_double, c_double, c_double,
                                         c_double, c_double, c_uint64, F, F, F]),
            "rto_sgd_update": (c_int, [F, F, c_size_t, c_double, F]),
            "rto_sgd_momentum_update": (c_int, [F, F, F, c_size_t, c_double, c_double, F, F]),
            "rto_fill_uniform": (None, [F, c_size_t, c_uint64, c_uint64, c_float, c_float]),
            "rto_fill_normal": (None, [F, c_size_t, c_uint64, c_uint64, c_float, c_float]),
            "rto_set_threads": (None, [c_int]), "rto_get_threads": (c_int, []),
            "rto_nn_adam_step": (None, [F, F, F, F, c_size_t, c_float, c_float, c_float,
                                        c_float, c_uint64, F, F, F]),
            "rto_nn_sgd_step": (None, [F, F, F, c_size_t, c_float, c_float, c_float, F, F]),
            "rto_broadcast_binary": (c_int, [c_int, F, sz, c_size_t, F, sz, c_size_t, F]),
            "rto_unrolled_sum_f32": (c_float, [F, c_size_t]),
            "rto_chain_sum_f32": (c_float, [F, c_size_t, c_float]),
            "rto_mse_loss": (c_double, [F, F, c_size_t]),
            "rto_l1_loss": (c_double, [F, F, c_size_t]),
            "rto_smooth_l1_loss": (c_double, [F, F, c_size_t, c_double]),
            "rto_bce_loss": (c_double, [F, F, c_size_t, c_double]),
            "rto_ce_loss": (c_double, [F, F, c_size_t, c_double]),
            "rto_relu_backward": (None, [F, F, F, c_size_t]),
            "rto_sigmoid_backward": (None, [F, F, F, c_size_t]),
            "rto_tanh_backward": (None, [F, F, F, c_size_t]),
            "rto_gelu_backward": (None, [F, F, F, c_size_t]),
            "rto_autograd_gelu": (None, [F, F, c_size_t]),
            "rto_sub_backward": (None, [F, F, F, c_size_t]),
            "rto_mul_backward": (None, [F, F, F, F, F, c_size_t]),
            "rto_div_backward": (None, [F, F, F, F, F, c_size_t]),
            "rto_fill_backward": (None, [c_float, F, c_size_t, c_int]),
            "rto_reduce_to_shape": (c_int, [F, sz, c_size_t, F, sz, c_size_t]),
        }
        for k, (r, a) in sig.items():
            fn = getattr(_lib, k)
            fn.restype = r
            fn.argtypes = a
    return _lib


def p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(c_void_p)


def uniform(n, seed, lo=-1.0, hi=1.0, offset=0):
    out = np.empty(n, dtype=np.float32)
    lib().rto_fill_uniform(p(out), n, seed, offset, lo, hi)
    return out


def normal(n, seed, mean=0.0, std=1.0, offset=0):
    out = np.empty(n, dtype=np.float32)
    lib().rto_fill_normal(p(out), n, seed, offset, mean, std)
    return out


def binary(name, a, b):
    out = np.empty_like(a)
    getattr(lib(), "rto_" + name)(p(a), p(b), p(out), a.size)
    return out


def unary(name, x, *extra):
    out = np.empty_like(x)
    fn = getattr(lib(), "rto_" + name)
    if extra:
        rc = fn(p(x), *extra, p(out), x.size)
    else:
        rc = fn(p(x), p(out), x.size)
    if rc not in (None, 0):
        raise ValueError(f"oracle {name} rc={rc}")
    return out


def scalar_op(name, x, s):
    out = np.empty_like(x)
    getattr(lib(), "rto_" + name)(p(x), s, p(out), x.size)
    return out


def fma(a, b, c):
    out = np.empty_like(a)
    lib().rto_fused_multiply_add(p(a), p(b), p(c), p(out), a.size)
    return out


def _shape(x):
    return (c_size_t * max(1, x.ndim))(*x.shape)


def softmax(x, dim):
    out = np.empty_like(x)
    rc = lib().rto_softmax(p(x), _shape(x), x.ndim, dim, p(out))
    if rc:
        raise ValueError(f"oracle softmax rc={rc}")
    return out


def reduce_dim(name, x, dim):
    shape = [d for i, d in enumerate(x.shape) if i != dim]
    out = np.empty(shape, dtype=np.float32)
    rc = getattr(lib(), f"rto_{name}_dim")(p(x), _shape(x), x.ndim, dim, p(out))
    if rc:
        raise ValueError(f"oracle {name}_dim rc={rc}")
    return out


def sum(x):  # noqa: A001
    return lib().rto_sum(p(x), x.size)


def scalar_reduce(name, x):
    v = c_double()
    rc = getattr(lib(), "rto_" + name)(p(x), x.size, ctypes.byref(v))
    return rc, v.value


def adamw(pp, g, m, v, lr, b1, b2, eps, wd, t):
    po, mo, vo = np.empty_like(pp), np.empty_like(pp), np.empty_like(pp)
    rc = lib().rto_adamw_update(p(pp), p(g), p(m), p(v), pp.size, lr, b1, b2, eps, wd, t,
                                p(po), p(mo), p(vo))
    return rc, po, mo, vo


def adam(pp, g, m, v, lr, b1, b2, eps, t):
    po, mo, vo = np.empty_like(pp), np.empty_like(pp), np.empty_like(pp)
    rc = lib().rto_adam_update(p(pp), p(g), p(m), p(v), pp.size, lr, b1, b2, eps, t,
                               p(po), p(mo), p(vo))
    return rc, po, mo, vo


def broadcast(op, a, b):
    """op in ("add", "sub", "mul", "div"); returns (rc, out)."""
    shape = np.broadcast_shapes(a.shape, b.shape) if _bok(a.shape, b.shape) else a.shape
    out = np.empty(shape, dtype=np.float32)
    rc = lib().rto_broadcast_binary(["add", "sub", "mul", "div"].index(op), p(a), _shape(a), a.ndim,
                                    p(b), _shape(b), b.ndim, p(out))
    return rc, out


def _bok(sa, sb):
    try:
        np.broadcast_shapes(sa, sb)
        return True
    except ValueError:
        return False


def nn_adam(pp, g, m, v, lr, b1, b2, eps, t):
    po, mo, vo = np.empty_like(pp), np.empty_like(pp), np.empty_like(pp)
    lib().rto_nn_adam_step(p(pp), p(g), p(m), p(v), pp.size, lr, b1, b2, eps, t, p(po), p(mo), p(vo))
    return po, mo, vo


def nn_sgd(pp, g, vel, lr, momentum, wd):
    po, vo = np.empty_like(pp), np.empty_like(pp)
    vel = vel if vel is not None else np.zeros_like(pp)
    lib().rto_nn_sgd_step(p(pp), p(g), p(vel), pp.size, lr, momentum, wd, p(po), p(vo))
    return po, vo


# ---- autograd backward (autograd/ops.rs) ----------------------------------
def grad_unary(name, g, saved):
    """name in relu, sigmoid, tanh, gelu; saved = input (relu, gelu) or output."""
    out = np.empty_like(g if name != "gelu" else saved)
    getattr(lib(), f"rto_{name}_backward")(p(g), p(saved), p(out), saved.size)
    return out


def autograd_gelu(x):
    out = np.empty_like(x)
    lib().rto_autograd_gelu(p(x), p(out), x.size)
    return out


def _opt(a):
    return p(a) if a is not None else None


def grad_binary(name, g, a=None, b=None, need_a=True, need_b=True):
    """name in add, sub, mul, div; returns (grad_a or None, grad_b or None)."""
    ga = np.empty_like(g) if need_a else None
    gb = np.empty_like(g) if need_b else None
    if name == "add":
        if ga is not None:
            ga[...] = g
        if gb is not None:
            gb[...] = g
    elif name == "sub":
        lib().rto_sub_backward(p(g), _opt(ga), _opt(gb), g.size)
    else:
        getattr(lib(), f"rto_{name}_backward")(p(g), p(a), p(b), _opt(ga), _opt(gb), g.size)
    return ga, gb


def fill_backward(g, shape, mean):
    out = np.empty(shape, dtype=np.float32)
    lib().rto_fill_backward(float(g), p(out), out.size, int(mean))
    return out


def reduce_to_shape(grad, shape):
    out = np.empty(shape, dtype=np.float32)
    o = np.empty(1, np.float32) if out.size == 0 else out
    rc = lib().rto_reduce_to_shape(p(grad), _shape(grad), grad.ndim, p(o),
                                   (c_size_t * max(1, len(shape)))(*shape), len(shape))
    return rc, out


# ---- losses (ops/loss.rs) -------------------------------------------------
def unrolled_sum_f32(x):
    """ndarray's sum() of a contiguous f32 array (eight chains), as an f32."""
    return np.float32(lib().rto_unrolled_sum_f32(p(x), x.size))


def chain_sum_f32(x, init=-0.0):
    """Iterator::sum of f32s from init, as an f32."""
    return np.float32(lib().rto_chain_sum_f32(p(x), x.size, init))


def loss(name, pred, targ, *param):
    """name in mse, l1, smooth_l1, bce, ce; returns the reference's f64."""
    return getattr(lib(), f"rto_{name}_loss")(p(pred), p(targ), pred.size, *map(float, param))
