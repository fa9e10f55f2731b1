"""rusttorch_b200 — rusttorch-core's data-parallel tensor hot path on B200.

The Python surface mirrors rusttorch's PyO3 module (rusttorch-py/src/lib.rs):
the same function names, argument meaning and error behaviour (every failure
raises ValueError, here the RusttorchError subclass carrying the TensorError
variant).  The difference is where the data lives: a `Tensor` here is a
float32 buffer in GPU memory, and every op is one call into
librusttorch_cuda.so (see include/rusttorch_cuda.h).  Ops are asynchronous on
the calling thread's stream; `to_numpy()` and the scalar reductions wait.
"""
from __future__ import annotations

import ctypes
from ctypes import c_double, c_void_p

import numpy as np

from . import _native
from ._native import F32, RusttorchError, check, lib

__all__ = [
    "Tensor", "RusttorchError", "version",
    "add", "sub", "mul", "div", "add_scalar", "mul_scalar", "add_mul_scalar",
    "fused_multiply_add", "add_simd", "mul_simd", "relu_simd", "mul_scalar_simd",
    "relu", "leaky_relu", "sigmoid", "tanh", "gelu", "swish", "elu", "selu", "mish",
    "softplus", "softsign", "softmax",
    "sum", "mean", "max", "min", "stats", "sum_dim", "mean_dim", "max_dim",
    "adam_update", "adamw_update", "sgd_update", "sgd_momentum_update",
    "add_broadcast", "sub_broadcast", "mul_broadcast", "div_broadcast",
    "nn_adam_step", "nn_sgd_step",
    "synchronize", "set_math_mode", "get_math_mode", "math_mode",
    "sharded_stats", "sharded_add_mul_scalar", "sharded_softmax", "sharded_sum_dim",
    "sharded_mean_dim", "sharded_max_dim", "sharded_adamw_update",
]


def version() -> str:
    return lib().rtc_version().decode()


def set_math_mode(mode: str) -> None:
    """"tolerance" (the default: within 1e-6 relative error or 4 ulp of the
    reference's glibc results, single-precision exp/tanh/log) or "exact"
    (glibc's expf/tanhf bit for bit) for the transcendental activations and
    softmax.  Process-wide (rtc_set_math_mode)."""
    code = {"tolerance": _native.MATH_TOLERANCE, "exact": _native.MATH_EXACT}.get(mode)
    if code is None:
        raise ValueError(f"math mode must be 'tolerance' or 'exact', not {mode!r}")
    check(lib().rtc_set_math_mode(code))


def get_math_mode() -> str:
    return "exact" if lib().rtc_get_math_mode() == _native.MATH_EXACT else "tolerance"


class math_mode:
    """Context manager: `with math_mode("exact"): ...` restores the previous
    mode on exit."""

    def __init__(self, mode: str):
        self.mode = mode

    def __enter__(self):
        self.before = get_math_mode()
        set_math_mode(self.mode)
        return self

    def __exit__(self, *exc):
        set_math_mode(self.before)


def synchronize() -> None:
    check(lib().rtc_synchronize())


class Tensor:
    """A C-contiguous float32 tensor in the memory of one GPU."""

    def __init__(self, shape, device: int = 0, *, ptr: int | None = None, owner=None):
        self._shape = tuple(int(d) for d in shape)
        self.device = int(device)
        self._owned = ptr is None
        self._owner = owner          # keeps a borrowed buffer alive
        if ptr is None:
            out = c_void_p()
            check(lib().rtc_malloc(self.device, self.nbytes, ctypes.byref(out)))
            ptr = out.value or 0
        self.ptr = int(ptr)
        self._desc = _native.Desc(self.ptr, self._shape, F32, self.device)

    # ---- construction (rusttorch-py/src/lib.rs:35-61) ---------------------
    @staticmethod
    def zeros(shape, device: int = 0) -> "Tensor":
        return Tensor.from_numpy(np.zeros(list(shape), dtype=np.float32), device)

    @staticmethod
    def ones(shape, device: int = 0) -> "Tensor":
        return Tensor.from_numpy(np.ones(list(shape), dtype=np.float32), device)

    @staticmethod
    def empty(shape, device: int = 0) -> "Tensor":
        return Tensor(shape, device)

    @staticmethod
    def from_numpy(array, device: int = 0) -> "Tensor":
        a = np.asarray(array)
        if a.dtype != np.float32:
            raise RusttorchError("only float32 arrays are supported", _native.UNSUPPORTED)
        if not a.flags.c_contiguous:
            raise ValueError("Array must be contiguous")
        t = Tensor(a.shape, device)
        if t.nbytes:
            check(lib().rtc_memcpy_h2d(t.device, c_void_p(t.ptr), a.ctypes.data_as(c_void_p),
                                       t.nbytes))
        return t

    @staticmethod
    def from_device_ptr(ptr: int, shape, device: int = 0, owner=None) -> "Tensor":
        """Borrow an existing device buffer (e.g. a torch tensor's data_ptr())."""
        return Tensor(shape, device, ptr=ptr, owner=owner)

    # ---- metadata (rusttorch-py/src/lib.rs:63-79) -------------------------
    def shape(self) -> list[int]:
        return list(self._shape)

    def ndim(self) -> int:
        return len(self._shape)

    def numel(self) -> int:
        n = 1
        for d in self._shape:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        return self.numel() * 4

    def __repr__(self) -> str:
        return f"Tensor(shape={list(self._shape)}, dtype=float32)"

    def to_numpy(self) -> np.ndarray:
        out = np.empty(self._shape, dtype=np.float32)
        if self.nbytes:
            check(lib().rtc_memcpy_d2h(self.device, out.ctypes.data_as(c_void_p),
                                       c_void_p(self.ptr), self.nbytes))
        return out

    @property
    def desc(self):
        """A by-reference rtc_tensor for a C-ABI call.  It holds this tensor
        (and so its device buffer) alive for as long as the reference itself
        is alive, so `Tensor.from_numpy(a).desc` passed straight to a call is
        safe: the temporary tensor is not freed before the call returns."""
        s = _native.RtcTensor.from_buffer_copy(self._desc.s)
        s._owner = self       # the copy -> the tensor; nothing points back
        return ctypes.byref(s)

    def __del__(self):
        try:
            if self._owned and self.ptr:
                lib().rtc_free(self.device, c_void_p(self.ptr))
                self.ptr = 0
        except Exception:
            pass


def _like(x: Tensor, shape=None) -> Tensor:
    return Tensor(x.shape() if shape is None else shape, x.device)


def _binary(fn, a: Tensor, b: Tensor) -> Tensor:
    out = _like(a)
    check(fn(a.desc, b.desc, out.desc))
    return out


def _unary(fn, x: Tensor, *extra) -> Tensor:
    out = _like(x)
    check(fn(x.desc, out.desc, *extra))
    return out


# ---- elementwise (rusttorch-py/src/lib.rs:83-123, :400-435) ----------------
def add(a: Tensor, b: Tensor) -> Tensor: return _binary(lib().rtc_add, a, b)
def mul(a: Tensor, b: Tensor) -> Tensor: return _binary(lib().rtc_mul, a, b)
def sub(a: Tensor, b: Tensor) -> Tensor: return _binary(lib().rtc_sub, a, b)
def div(a: Tensor, b: Tensor) -> Tensor: return _binary(lib().rtc_div, a, b)
def add_simd(a: Tensor, b: Tensor) -> Tensor: return _binary(lib().rtc_add_simd, a, b)
def mul_simd(a: Tensor, b: Tensor) -> Tensor: return _binary(lib().rtc_mul_simd, a, b)


def add_scalar(t: Tensor, scalar: float) -> Tensor:
    out = _like(t)
    check(lib().rtc_add_scalar(t.desc, float(scalar), out.desc))
    return out


def mul_scalar(t: Tensor, scalar: float) -> Tensor:
    out = _like(t)
    check(lib().rtc_mul_scalar(t.desc, float(scalar), out.desc))
    return out


def mul_scalar_simd(t: Tensor, scalar: float) -> Tensor:
    out = _like(t)
    check(lib().rtc_mul_scalar_simd(t.desc, float(scalar), out.desc))
    return out


def add_mul_scalar(a: Tensor, b: Tensor, scalar: float) -> Tensor:
    """mul_scalar(add(a, b), scalar) in one pass over memory."""
    out = _like(a)
    check(lib().rtc_add_mul_scalar(a.desc, b.desc, float(scalar), out.desc))
    return out


def fused_multiply_add(a: Tensor, b: Tensor, c: Tensor) -> Tensor:
    out = _like(a)
    check(lib().rtc_fused_multiply_add(a.desc, b.desc, c.desc, out.desc))
    return out


# ---- activations (rusttorch-py/src/lib.rs:126-208) --------------------------
def relu(t: Tensor) -> Tensor: return _unary(lib().rtc_relu, t)
def relu_simd(t: Tensor) -> Tensor: return _unary(lib().rtc_relu_simd, t)
def sigmoid(t: Tensor) -> Tensor: return _unary(lib().rtc_sigmoid, t)
def tanh(t: Tensor) -> Tensor: return _unary(lib().rtc_tanh, t)
def gelu(t: Tensor) -> Tensor: return _unary(lib().rtc_gelu, t)
def swish(t: Tensor) -> Tensor: return _unary(lib().rtc_swish, t)
def selu(t: Tensor) -> Tensor: return _unary(lib().rtc_selu, t)
def mish(t: Tensor) -> Tensor: return _unary(lib().rtc_mish, t)
def softplus(t: Tensor) -> Tensor: return _unary(lib().rtc_softplus, t)
def softsign(t: Tensor) -> Tensor: return _unary(lib().rtc_softsign, t)
def leaky_relu(t: Tensor, alpha: float) -> Tensor: return _unary(lib().rtc_leaky_relu, t, float(alpha))
def elu(t: Tensor, alpha: float) -> Tensor: return _unary(lib().rtc_elu, t, float(alpha))


def softmax(t: Tensor, dim: int) -> Tensor:
    out = _like(t)
    check(lib().rtc_softmax(t.desc, int(dim), out.desc))
    return out


# ---- reductions (rusttorch-py/src/lib.rs:234-242; core reduction.rs) -------
def _scalar(fn, t: Tensor) -> float:
    v = c_double()
    check(fn(t.desc, ctypes.byref(v)))
    return v.value


def sum(t: Tensor) -> float: return _scalar(lib().rtc_sum, t)     # noqa: A001
def mean(t: Tensor) -> float: return _scalar(lib().rtc_mean, t)
def max(t: Tensor) -> float: return _scalar(lib().rtc_max, t)     # noqa: A001
def min(t: Tensor) -> float: return _scalar(lib().rtc_min, t)     # noqa: A001


def stats(t: Tensor) -> tuple[float, float, float, float]:
    """(sum, mean, max, min) from one pass."""
    v = (c_double * 4)()
    check(lib().rtc_stats(t.desc, v))
    return tuple(v)


def _dim(fn, t: Tensor, dim: int) -> Tensor:
    dim = int(dim)
    shape = [d for i, d in enumerate(t.shape()) if i != dim] if 0 <= dim < t.ndim() else []
    out = _like(t, shape)
    check(fn(t.desc, dim, out.desc))
    return out


def sum_dim(t: Tensor, dim: int) -> Tensor: return _dim(lib().rtc_sum_dim, t, dim)
def mean_dim(t: Tensor, dim: int) -> Tensor: return _dim(lib().rtc_mean_dim, t, dim)
def max_dim(t: Tensor, dim: int) -> Tensor: return _dim(lib().rtc_max_dim, t, dim)


# ---- optimizers (rusttorch-py/src/lib.rs:278-369) --------------------------
def adam_update(params, gradients, m, v, learning_rate, beta1, beta2, epsilon, timestep):
    po, mo, vo = _like(params), _like(params), _like(params)
    check(lib().rtc_adam_update(params.desc, gradients.desc, m.desc, v.desc, float(learning_rate),
                                float(beta1), float(beta2), float(epsilon), int(timestep),
                                po.desc, mo.desc, vo.desc))
    return po, mo, vo


def adamw_update(params, gradients, m, v, learning_rate, beta1, beta2, epsilon, weight_decay,
                 timestep):
    po, mo, vo = _like(params), _like(params), _like(params)
    check(lib().rtc_adamw_update(params.desc, gradients.desc, m.desc, v.desc,
                                 float(learning_rate), float(beta1), float(beta2), float(epsilon),
                                 float(weight_decay), int(timestep), po.desc, mo.desc, vo.desc))
    return po, mo, vo


def sgd_update(params, gradients, learning_rate):
    po = _like(params)
    check(lib().rtc_sgd_update(params.desc, gradients.desc, float(learning_rate), po.desc))
    return po


def sgd_momentum_update(params, gradients, velocity, learning_rate, momentum):
    po, vo = _like(params), _like(params)
    check(lib().rtc_sgd_momentum_update(params.desc, gradients.desc, velocity.desc,
                                        float(learning_rate), float(momentum), po.desc, vo.desc))
    return po, vo


# ---- broadcasting (rusttorch-py/src/lib.rs:372-398; core ops/broadcast.rs) ----
def _bshape(a: Tensor, b: Tensor):
    try:
        return list(np.broadcast_shapes(tuple(a.shape()), tuple(b.shape())))
    except ValueError:
        return a.shape()          # the library reports the BroadcastError


def _bcast(fn, a: Tensor, b: Tensor) -> Tensor:
    out = _like(a, _bshape(a, b))
    check(fn(a.desc, b.desc, out.desc))
    return out


def add_broadcast(a: Tensor, b: Tensor) -> Tensor: return _bcast(lib().rtc_add_broadcast, a, b)
def sub_broadcast(a: Tensor, b: Tensor) -> Tensor: return _bcast(lib().rtc_sub_broadcast, a, b)
def mul_broadcast(a: Tensor, b: Tensor) -> Tensor: return _bcast(lib().rtc_mul_broadcast, a, b)
def div_broadcast(a: Tensor, b: Tensor) -> Tensor: return _bcast(lib().rtc_div_broadcast, a, b)


# ---- nn optimizers (core nn/optim.rs), one parameter per call ---------------
def nn_adam_step(params, grads, m, v, lr, beta1, beta2, eps, t):
    """nn::Adam::step for one parameter; t counts steps from 1."""
    po, mo, vo = _like(params), _like(params), _like(params)
    check(lib().rtc_nn_adam_step(params.desc, grads.desc, m.desc, v.desc, float(lr),
                                 float(beta1), float(beta2), float(eps), int(t), po.desc,
                                 mo.desc, vo.desc))
    return po, mo, vo


def nn_sgd_step(params, grads, velocity, lr, momentum=0.0, weight_decay=0.0):
    """nn::SGD::step for one parameter; returns (params', velocity')
    (velocity' is None without momentum)."""
    po = _like(params)
    if momentum > 0.0:
        vo = _like(params)
        check(lib().rtc_nn_sgd_step(params.desc, grads.desc, velocity.desc, float(lr),
                                    float(momentum), float(weight_decay), po.desc, vo.desc))
        return po, vo
    check(lib().rtc_nn_sgd_step(params.desc, grads.desc, None, float(lr), float(momentum),
                                float(weight_decay), po.desc, None))
    return po, None


# ---- autograd backward (core autograd/ops.rs GradFn::backward) -------------
# Each returns what the reference's backward returns for that input; pass
# need_a / need_b False where the reference's operand does not require grad
# (its `None`).
def relu_backward(grad_output: Tensor, input: Tensor) -> Tensor:
    out = _like(grad_output)
    check(lib().rtc_relu_backward(grad_output.desc, input.desc, out.desc))
    return out


def sigmoid_backward(grad_output: Tensor, output: Tensor) -> Tensor:
    out = _like(grad_output)
    check(lib().rtc_sigmoid_backward(grad_output.desc, output.desc, out.desc))
    return out


def tanh_backward(grad_output: Tensor, output: Tensor) -> Tensor:
    out = _like(grad_output)
    check(lib().rtc_tanh_backward(grad_output.desc, output.desc, out.desc))
    return out


def gelu_backward(grad_output: Tensor, input: Tensor) -> Tensor:
    out = _like(input)
    check(lib().rtc_gelu_backward(grad_output.desc, input.desc, out.desc))
    return out


def autograd_gelu(x: Tensor) -> Tensor:
    """autograd's own GELU forward (it rounds differently from gelu)."""
    out = _like(x)
    check(lib().rtc_autograd_gelu(x.desc, out.desc))
    return out


def _pair_out(g: Tensor, need_a: bool, need_b: bool):
    return (_like(g) if need_a else None), (_like(g) if need_b else None)


def _d(t):
    return t.desc if t is not None else None


def add_backward(grad_output: Tensor, need_a=True, need_b=True):
    ga, gb = _pair_out(grad_output, need_a, need_b)
    check(lib().rtc_add_backward(grad_output.desc, _d(ga), _d(gb)))
    return ga, gb


def sub_backward(grad_output: Tensor, need_a=True, need_b=True):
    ga, gb = _pair_out(grad_output, need_a, need_b)
    check(lib().rtc_sub_backward(grad_output.desc, _d(ga), _d(gb)))
    return ga, gb


def mul_backward(grad_output: Tensor, a: Tensor, b: Tensor, need_a=True, need_b=True):
    ga, gb = _pair_out(grad_output, need_a, need_b)
    check(lib().rtc_mul_backward(grad_output.desc, a.desc, b.desc, _d(ga), _d(gb)))
    return ga, gb


def div_backward(grad_output: Tensor, a: Tensor, b: Tensor, need_a=True, need_b=True):
    ga, gb = _pair_out(grad_output, need_a, need_b)
    check(lib().rtc_div_backward(grad_output.desc, a.desc, b.desc, _d(ga), _d(gb)))
    return ga, gb


def sum_backward(grad_output: Tensor, input_shape) -> Tensor:
    out = Tensor(list(input_shape), device=grad_output.device)
    check(lib().rtc_sum_backward(grad_output.desc, out.desc))
    return out


def mean_backward(grad_output: Tensor, input_shape) -> Tensor:
    out = Tensor(list(input_shape), device=grad_output.device)
    check(lib().rtc_mean_backward(grad_output.desc, out.desc))
    return out


def broadcast_add_backward(grad_output: Tensor, a_shape, b_shape, need_a=True, need_b=True):
    ga = Tensor(list(a_shape), device=grad_output.device) if need_a else None
    gb = Tensor(list(b_shape), device=grad_output.device) if need_b else None
    check(lib().rtc_broadcast_add_backward(grad_output.desc, _d(ga), _d(gb)))
    return ga, gb


# ---- loss functions (core ops/loss.rs): Python floats, like rusttorch's f64 --
def _loss(fn, predictions: Tensor, targets: Tensor, *args) -> float:
    v = ctypes.c_double()
    check(fn(predictions.desc, targets.desc, *args, ctypes.byref(v)))
    return v.value


def mse_loss(predictions: Tensor, targets: Tensor) -> float:
    return _loss(lib().rtc_mse_loss, predictions, targets)


def l1_loss(predictions: Tensor, targets: Tensor) -> float:
    return _loss(lib().rtc_l1_loss, predictions, targets)


def smooth_l1_loss(predictions: Tensor, targets: Tensor, beta: float = 1.0) -> float:
    return _loss(lib().rtc_smooth_l1_loss, predictions, targets, float(beta))


def binary_cross_entropy_loss(predictions: Tensor, targets: Tensor, epsilon: float = 1e-7) -> float:
    return _loss(lib().rtc_binary_cross_entropy_loss, predictions, targets, float(epsilon))


def cross_entropy_loss(predictions: Tensor, targets: Tensor, epsilon: float = 1e-7) -> float:
    return _loss(lib().rtc_cross_entropy_loss, predictions, targets, float(epsilon))


# ---- one process, several GPUs ---------------------------------------------
def sharded_stats(shards) -> tuple[float, float, float, float]:
    """(sum, mean, max, min) of the concatenation of `shards` (Tensors, each
    on its own GPU or not), every shard summarised on its device at once."""
    shards = list(shards)
    arr = (_native.RtcTensor * (len(shards) or 1))()
    for i, t in enumerate(shards):
        arr[i] = t._desc.s
    out = (c_double * 4)()
    check(lib().rtc_sharded_stats(arr, len(shards), out))
    return out[0], out[1], out[2], out[3]


def _desc_array(tensors):
    arr = (_native.RtcTensor * (len(tensors) or 1))()
    for i, t in enumerate(tensors):
        arr[i] = t._desc.s
    return arr


def _like_shards(shards, shapes=None):
    return [_like(t, shapes[i] if shapes else None) for i, t in enumerate(shards)]


def sharded_add_mul_scalar(a, b, scalar: float):
    """mul_scalar(add(a, b), scalar) of a tensor split into shards (lists of
    Tensors, shard i of a and b on one GPU): one new Tensor per shard."""
    a, b = list(a), list(b)
    if len(a) != len(b):
        raise ValueError("a and b must have the same number of shards")
    out = _like_shards(a)
    check(lib().rtc_sharded_add_mul_scalar(_desc_array(a), _desc_array(b), float(scalar),
                                           _desc_array(out), len(a)))
    return out


def sharded_softmax(shards, dim: int):
    """softmax along `dim` of row blocks (the shards split axis 0)."""
    shards = list(shards)
    out = _like_shards(shards)
    check(lib().rtc_sharded_softmax(_desc_array(shards), dim, _desc_array(out), len(shards)))
    return out


def _sharded_dim(fn, shards, dim: int):
    shards = list(shards)
    dim = int(dim)
    out = _like_shards(shards, [[d for k, d in enumerate(t.shape()) if k != dim]
                                if 0 <= dim < t.ndim() else [] for t in shards])
    check(fn(_desc_array(shards), dim, _desc_array(out), len(shards)))
    return out


def sharded_sum_dim(shards, dim: int):
    """sum_dim of each shard on its own GPU (the shards split an axis other
    than dim: column blocks for dim 0, row blocks for the last axis)."""
    return _sharded_dim(lib().rtc_sharded_sum_dim, shards, dim)


def sharded_mean_dim(shards, dim: int):
    return _sharded_dim(lib().rtc_sharded_mean_dim, shards, dim)


def sharded_max_dim(shards, dim: int):
    return _sharded_dim(lib().rtc_sharded_max_dim, shards, dim)


def sharded_adamw_update(params, grads, m, v, learning_rate, beta1, beta2, epsilon, weight_decay,
                         timestep):
    """adamw_update of every shard, in place (params, m, v are updated)."""
    params, grads, m, v = list(params), list(grads), list(m), list(v)
    if not len(params) == len(grads) == len(m) == len(v):
        raise ValueError("params, grads, m and v must have the same number of shards")
    check(lib().rtc_sharded_adamw_update(_desc_array(params), _desc_array(grads), _desc_array(m),
                                         _desc_array(v), learning_rate, beta1, beta2, epsilon,
                                         weight_decay, int(timestep), len(params)))
