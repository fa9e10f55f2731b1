"""ctypes binding of librusttorch_cuda.so (include/rusttorch_cuda.h).

The library is the product: there is no Python or CPU fallback.  If it has
not been built, every call raises instead of silently computing elsewhere.
"""
from __future__ import annotations

import ctypes
import re
from ctypes import (POINTER, Structure, c_bool, c_char_p, c_double, c_float, c_int, c_size_t,
                    c_uint64, c_void_p)
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "librusttorch_cuda.so"
HEADER_PATH = PKG.parent / "include" / "rusttorch_cuda.h"

# math modes (rtc_set_math_mode)
MATH_TOLERANCE, MATH_EXACT = 0, 1
# peer-memory exchange (rtc_peer_allreduce_sum_f64)
IPC_HANDLE_BYTES, PEER_MAX_RANKS = 64, 8
# dtype codes and status codes (rusttorch_cuda.h)
F32, F64, I32, I64 = 0, 1, 2, 3
OK, SHAPE_MISMATCH, DTYPE_MISMATCH, EMPTY_TENSOR, INVALID_DIMENSION, INVALID_ARGUMENT, \
    SIZE_OVERFLOW, UNSUPPORTED, BACKEND_ERROR, BROADCAST_ERROR = range(10)
STATUS_NAMES = {
    OK: "Ok", SHAPE_MISMATCH: "ShapeMismatch", DTYPE_MISMATCH: "DTypeMismatch",
    EMPTY_TENSOR: "EmptyTensor", INVALID_DIMENSION: "InvalidDimension",
    INVALID_ARGUMENT: "InvalidArgument", SIZE_OVERFLOW: "SizeOverflow",
    UNSUPPORTED: "Unsupported", BACKEND_ERROR: "BackendError", BROADCAST_ERROR: "BroadcastError",
}


class RtcTensor(Structure):
    _fields_ = [
        ("data", c_void_p),
        ("shape", POINTER(c_size_t)),
        ("strides", POINTER(c_size_t)),
        ("ndim", c_size_t),
        ("numel", c_size_t),
        ("dtype", c_int),
        ("device", c_int),
    ]


class RtcResult(Structure):
    _fields_ = [("success", c_bool), ("error_msg", c_void_p), ("code", c_int)]


class ShardSummary(Structure):
    """rtc_shard_summary (include/rusttorch_cuda.h)."""
    _fields_ = [("sum", c_double), ("count", c_uint64), ("max", c_float),
                ("min_nonnan", c_float), ("max_kind", ctypes.c_int32),
                ("first_nan", ctypes.c_int32)]


class RusttorchError(ValueError):
    """A failed call.  rusttorch-py maps every TensorError to ValueError
    (rusttorch-py/src/lib.rs:23-25); `code` names the TensorError variant."""

    def __init__(self, message: str, code: int):
        super().__init__(message)
        self.code = code
        self.kind = STATUS_NAMES.get(code, str(code))


T = POINTER(RtcTensor)
_SIGNATURES = {
    "rtc_version": (c_char_p, []),
    "rtc_init": (RtcResult, []),
    "rtc_cleanup": (None, []),
    "rtc_free_error_message": (None, [c_void_p]),
    "rtc_set_stream": (RtcResult, [c_void_p]),
    "rtc_get_stream": (c_void_p, []),
    "rtc_synchronize": (RtcResult, []),
    "rtc_device_count": (c_int, []),
    "rtc_set_device": (RtcResult, [c_int]),
    "rtc_get_device": (c_int, []),
    "rtc_malloc": (RtcResult, [c_int, c_size_t, POINTER(c_void_p)]),
    "rtc_free": (RtcResult, [c_int, c_void_p]),
    "rtc_memcpy_h2d": (RtcResult, [c_int, c_void_p, c_void_p, c_size_t]),
    "rtc_memcpy_d2h": (RtcResult, [c_int, c_void_p, c_void_p, c_size_t]),
    "rtc_host_alloc": (RtcResult, [c_size_t, POINTER(c_void_p)]),
    "rtc_host_free": (RtcResult, [c_void_p]),
    "rtc_fill_uniform": (RtcResult, [T, c_uint64, c_uint64, c_float, c_float]),
    "rtc_fill_normal": (RtcResult, [T, c_uint64, c_uint64, c_float, c_float]),
    "rtc_add": (RtcResult, [T, T, T]),
    "rtc_mul": (RtcResult, [T, T, T]),
    "rtc_sub": (RtcResult, [T, T, T]),
    "rtc_div": (RtcResult, [T, T, T]),
    "rtc_add_scalar": (RtcResult, [T, c_float, T]),
    "rtc_mul_scalar": (RtcResult, [T, c_float, T]),
    "rtc_add_mul_scalar": (RtcResult, [T, T, c_float, T]),
    "rtc_fused_multiply_add": (RtcResult, [T, T, T, T]),
    "rtc_add_simd": (RtcResult, [T, T, T]),
    "rtc_mul_simd": (RtcResult, [T, T, T]),
    "rtc_relu_simd": (RtcResult, [T, T]),
    "rtc_mul_scalar_simd": (RtcResult, [T, c_float, T]),
    "rtc_relu": (RtcResult, [T, T]),
    "rtc_leaky_relu": (RtcResult, [T, T, c_float]),
    "rtc_sigmoid": (RtcResult, [T, T]),
    "rtc_tanh": (RtcResult, [T, T]),
    "rtc_gelu": (RtcResult, [T, T]),
    "rtc_swish": (RtcResult, [T, T]),
    "rtc_elu": (RtcResult, [T, T, c_float]),
    "rtc_selu": (RtcResult, [T, T]),
    "rtc_mish": (RtcResult, [T, T]),
    "rtc_softplus": (RtcResult, [T, T]),
    "rtc_softsign": (RtcResult, [T, T]),
    "rtc_softmax": (RtcResult, [T, c_size_t, T]),
    "rtc_sum": (RtcResult, [T, POINTER(c_double)]),
    "rtc_mean": (RtcResult, [T, POINTER(c_double)]),
    "rtc_max": (RtcResult, [T, POINTER(c_double)]),
    "rtc_min": (RtcResult, [T, POINTER(c_double)]),
    "rtc_stats": (RtcResult, [T, POINTER(c_double)]),
    "rtc_sum_device": (RtcResult, [T, c_void_p]),
    "rtc_sum_device_noalloc": (RtcResult, [T, c_void_p]),
    "rtc_sum_dim": (RtcResult, [T, c_size_t, T]),
    "rtc_mean_dim": (RtcResult, [T, c_size_t, T]),
    "rtc_max_dim": (RtcResult, [T, c_size_t, T]),
    "rtc_adam_update": (RtcResult, [T, T, T, T, c_double, c_double, c_double, c_double, c_uint64,
                                    T, T, T]),
    "rtc_adamw_update": (RtcResult, [T, T, T, T, c_double, c_double, c_double, c_double,
                                     c_double, c_uint64, T, T, T]),
    "rtc_sgd_update": (RtcResult, [T, T, c_double, T]),
    "rtc_sgd_momentum_update": (RtcResult, [T, T, T, c_double, c_double, T, T]),
    "rtc_shard_summary_local": (RtcResult, [T, POINTER(ShardSummary)]),
    "rtc_shard_combine": (RtcResult, [POINTER(ShardSummary), c_size_t, POINTER(c_double)]),
    "rtc_sharded_stats": (RtcResult, [POINTER(RtcTensor), c_size_t, POINTER(c_double)]),
    "rtc_sharded_add_mul_scalar": (RtcResult, [T, T, c_float, T, c_size_t]),
    "rtc_sharded_softmax": (RtcResult, [T, c_size_t, T, c_size_t]),
    "rtc_sharded_sum_dim": (RtcResult, [T, c_size_t, T, c_size_t]),
    "rtc_sharded_mean_dim": (RtcResult, [T, c_size_t, T, c_size_t]),
    "rtc_sharded_max_dim": (RtcResult, [T, c_size_t, T, c_size_t]),
    "rtc_sharded_adamw_update": (RtcResult, [T, T, T, T, c_double, c_double, c_double, c_double,
                                             c_double, c_uint64, c_size_t]),
    "rtc_ipc_handle": (RtcResult, [c_int, c_void_p, c_void_p]),
    "rtc_ipc_open": (RtcResult, [c_int, c_void_p, POINTER(c_void_p)]),
    "rtc_ipc_close": (RtcResult, [c_int, c_void_p]),
    "rtc_peer_slot_bytes": (c_size_t, [c_int]),
    "rtc_peer_allreduce_sum_f64": (RtcResult, [c_int, c_void_p, POINTER(c_void_p), c_int, c_int,
                                               c_uint64, c_void_p]),
    "rtc_selftest_bounded_wait": (RtcResult, []),
    "rtc_selftest_ordered_sum": (RtcResult, [T, c_int, c_float, POINTER(c_float)]),
    "rtc_add_broadcast": (RtcResult, [T, T, T]),
    "rtc_sub_broadcast": (RtcResult, [T, T, T]),
    "rtc_mul_broadcast": (RtcResult, [T, T, T]),
    "rtc_div_broadcast": (RtcResult, [T, T, T]),
    "rtc_nn_adam_step": (RtcResult, [T, T, T, T, c_float, c_float, c_float, c_float, c_uint64,
                                     T, T, T]),
    "rtc_nn_sgd_step": (RtcResult, [T, T, T, c_float, c_float, c_float, T, T]),
    "rtc_mse_loss": (RtcResult, [T, T, POINTER(c_double)]),
    "rtc_l1_loss": (RtcResult, [T, T, POINTER(c_double)]),
    "rtc_smooth_l1_loss": (RtcResult, [T, T, c_double, POINTER(c_double)]),
    "rtc_binary_cross_entropy_loss": (RtcResult, [T, T, c_double, POINTER(c_double)]),
    "rtc_cross_entropy_loss": (RtcResult, [T, T, c_double, POINTER(c_double)]),
    "rtc_relu_backward": (RtcResult, [T, T, T]),
    "rtc_sigmoid_backward": (RtcResult, [T, T, T]),
    "rtc_tanh_backward": (RtcResult, [T, T, T]),
    "rtc_gelu_backward": (RtcResult, [T, T, T]),
    "rtc_autograd_gelu": (RtcResult, [T, T]),
    "rtc_add_backward": (RtcResult, [T, T, T]),
    "rtc_sub_backward": (RtcResult, [T, T, T]),
    "rtc_mul_backward": (RtcResult, [T, T, T, T, T]),
    "rtc_div_backward": (RtcResult, [T, T, T, T, T]),
    "rtc_sum_backward": (RtcResult, [T, T]),
    "rtc_mean_backward": (RtcResult, [T, T]),
    "rtc_broadcast_add_backward": (RtcResult, [T, T, T]),
    "rtc_relu_f32": (RtcResult, [c_void_p, c_void_p, c_size_t]),
    "rtc_add_f32": (RtcResult, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "rtc_mul_f32": (RtcResult, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "rtc_probe_stream": (RtcResult, [c_int, c_void_p, c_void_p, c_size_t, c_int, c_int, c_int]),
    "rtc_set_math_mode": (RtcResult, [c_int]),
    "rtc_get_math_mode": (c_int, []),
    "rtc_selftest_fastmath": (RtcResult, [c_int, c_void_p, c_void_p, c_size_t]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m rusttorch_b200.build` "
                "(there is no CPU fallback)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def header_functions() -> list[str]:
    """Names of the functions include/rusttorch_cuda.h declares."""
    text = HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rtc_\w+)\s*\(", text)))


def check(res: RtcResult) -> None:
    """Raise RusttorchError for a failed rtc_result (and free its message)."""
    if res.success:
        return
    msg = ctypes.string_at(res.error_msg).decode() if res.error_msg else "unknown error"
    if res.error_msg:
        lib().rtc_free_error_message(res.error_msg)
    raise RusttorchError(msg, res.code)


class Desc:
    """An rtc_tensor descriptor that keeps its shape array alive."""

    __slots__ = ("shape_arr", "s")

    def __init__(self, ptr: int, shape, dtype: int = F32, device: int = 0):
        shape = [int(d) for d in shape]
        numel = 1
        for d in shape:
            numel *= d
        self.shape_arr = (c_size_t * max(1, len(shape)))(*shape)
        self.s = RtcTensor(c_void_p(ptr or None), self.shape_arr, None, len(shape), numel, dtype,
                           device)

    @property
    def ref(self):
        return ctypes.byref(self.s)
