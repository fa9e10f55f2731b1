"""The C ABI on the CPU: loading, exported symbols, and host-side validation.

Validation runs before any CUDA call, so every error path below works without
a GPU.  The expected texts are rusttorch's TensorError Display strings
(rusttorch-core/src/error.rs:69-160) for the same calls on the reference.
Descriptors point at a dummy address: nothing is dereferenced on these paths.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import pytest

from rusttorch_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]

DUMMY = 0x1000


def desc(shape, dtype=N.F32, device=0, ptr=DUMMY):
    return N.Desc(ptr, shape, dtype, device)


def call(name, *args):
    res = getattr(N.lib(), name)(*args)
    if res.success:
        return None
    msg = ctypes.string_at(res.error_msg).decode()
    N.lib().rtc_free_error_message(res.error_msg)
    return res.code, msg


def test_library_loads_and_reports_version():
    assert N.lib().rtc_version().decode() == "0.1.0"


def test_every_header_symbol_is_exported():
    names = N.header_functions()
    assert len(names) >= 50
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:          # and ctypes resolves each of them
        getattr(N.lib(), n)


def test_binding_table_covers_header():
    assert set(N.header_functions()) <= set(N._SIGNATURES)


def test_mixing_host_and_device_is_an_error():
    host = N.Desc(DUMMY, [4], N.F32, -1)
    dev = N.Desc(DUMMY, [4], N.F32, 0)
    code, msg = call("rtc_add", host.ref, dev.ref, host.ref)
    assert code == N.INVALID_ARGUMENT and "host-memory" in msg


def test_add_dtype_checked_before_shape():            # elementwise.rs:15-28
    a, b, o = desc([2, 2]), desc([3, 3], N.F64), desc([2, 2])
    assert call("rtc_add", a.ref, b.ref, o.ref) == (
        N.DTYPE_MISMATCH, "Data type mismatch in element-wise addition: expected Float32, got Float64")


def test_add_shape_mismatch():                         # elementwise.rs:288-298
    a, b, o = desc([2, 2]), desc([3, 3]), desc([2, 2])
    assert call("rtc_add", a.ref, b.ref, o.ref) == (
        N.SHAPE_MISMATCH, "Shape mismatch in element-wise addition: expected [2, 2], got [3, 3]")


def test_div_requires_float():                         # elementwise.rs:178-183
    a, b, o = desc([4], N.I32), desc([4], N.I32), desc([4], N.I32)
    assert call("rtc_div", a.ref, b.ref, o.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'dtype': Division requires floating-point tensors")


def test_int_add_is_unsupported_after_reference_checks():
    a, b, o = desc([4], N.I32), desc([4], N.I32), desc([4], N.I32)
    code, msg = call("rtc_add", a.ref, b.ref, o.ref)
    assert code == N.UNSUPPORTED and "int32" in msg


def test_sigmoid_int_error():                          # activation.rs:417-426
    x, o = desc([2, 2], N.I32), desc([2, 2], N.I32)
    assert call("rtc_sigmoid", x.ref, o.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'dtype': Sigmoid requires floating-point tensors")


def test_softmax_dim_out_of_range():                   # activation.rs:428-437
    x, o = desc([2, 3]), desc([2, 3])
    assert call("rtc_softmax", x.ref, 5, o.ref) == (
        N.INVALID_DIMENSION, "Invalid dimension in softmax: 5 (max: 1)")


def test_elu_negative_alpha():                          # activation.rs:481-490
    x, o = desc([1]), desc([1])
    assert call("rtc_elu", x.ref, o.ref, ctypes.c_float(-0.5)) == (
        N.INVALID_ARGUMENT, "Invalid argument 'alpha': Alpha must be positive")


@pytest.mark.parametrize("name", ["rtc_mean", "rtc_max", "rtc_min"])
def test_empty_reductions(name):                        # reduction.rs:198-236
    x = desc([0], ptr=0)
    v = ctypes.c_double()
    op = name[4:]
    assert call(name, x.ref, ctypes.byref(v)) == (N.EMPTY_TENSOR,
                                                  f"Cannot perform {op} on empty tensor")


def test_sum_of_empty_is_zero_without_gpu():            # reduction.rs:210-214
    x = desc([0], ptr=0)
    v = ctypes.c_double(123.0)
    assert call("rtc_sum", x.ref, ctypes.byref(v)) is None
    assert v.value == 0.0


def test_sum_dim_out_of_range():                        # reduction.rs:239-247
    x, o = desc([2, 2]), desc([2])
    assert call("rtc_sum_dim", x.ref, 5, o.ref) == (
        N.INVALID_DIMENSION, "Invalid dimension in sum_dim: 5 (max: 1)")


def test_mean_dim_of_empty_axis():
    # The reference panics here (mean_axis(..).unwrap() on a zero-length axis);
    # the C ABI reports EmptyTensor instead.
    x, o = desc([3, 0], ptr=0), desc([3])
    assert call("rtc_mean_dim", x.ref, 1, o.ref) == (N.EMPTY_TENSOR,
                                                     "Cannot perform mean_dim on empty tensor")


def test_adam_checks_in_reference_order():              # optimizer.rs:219-271
    p, g3, o = desc([3]), desc([2]), desc([3])
    assert call("rtc_adam_update", p.ref, g3.ref, p.ref, p.ref, 0.001, 0.9, 0.999, 1e-8, 1,
                o.ref, o.ref, o.ref) == (
        N.SHAPE_MISMATCH,
        "Shape mismatch in adam_update (params vs gradients): expected [3], got [2]")
    assert call("rtc_adam_update", p.ref, p.ref, p.ref, p.ref, -0.001, 0.9, 0.999, 1e-8, 1,
                o.ref, o.ref, o.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'learning_rate': must be positive, got -0.001")
    assert call("rtc_adam_update", p.ref, p.ref, p.ref, p.ref, 0.001, 1.5, 0.999, 1e-8, 1,
                o.ref, o.ref, o.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'beta1': must be in (0, 1), got 1.5")
    assert call("rtc_adam_update", p.ref, p.ref, p.ref, p.ref, 0.001, 0.9, 0.999, 0.0, 1,
                o.ref, o.ref, o.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'epsilon': must be positive, got 0")
    assert call("rtc_adam_update", p.ref, p.ref, p.ref, p.ref, 0.001, 0.9, 0.999, 1e-8, 0,
                o.ref, o.ref, o.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'timestep': must be >= 1")
    i = desc([3], N.I32)
    assert call("rtc_adam_update", i.ref, i.ref, i.ref, i.ref, 0.001, 0.9, 0.999, 1e-8, 1,
                i.ref, i.ref, i.ref) == (
        N.DTYPE_MISMATCH,
        "Data type mismatch in adam_update (only floating-point supported): expected float32 or"
        " float64, got int32")


def test_adamw_weight_decay_checked_first():            # optimizer.rs:392-397
    p, g2 = desc([3]), desc([2])
    assert call("rtc_adamw_update", p.ref, g2.ref, p.ref, p.ref, 0.001, 0.9, 0.999, 1e-8, -0.01,
                1, p.ref, p.ref, p.ref) == (
        N.INVALID_ARGUMENT, "Invalid argument 'weight_decay': must be non-negative, got -0.01")


def test_rust_float_display():
    # Rust prints f64 in positional notation with the shortest round-trip digits.
    for v, s in [(1e-8, "0.00000001"), (-0.1, "-0.1"), (1.0, "1"), (2.5e20, "250000000000000000000")]:
        p = desc([1])
        got = call("rtc_adam_update", p.ref, p.ref, p.ref, p.ref, 0.001, 0.9, 0.999, -abs(v) if v > 0 else v,
                   1, p.ref, p.ref, p.ref)
        expect = s if s.startswith("-") else "-" + s
        assert got == (N.INVALID_ARGUMENT, f"Invalid argument 'epsilon': must be positive, got {expect}")


def test_descriptor_sanity():
    bad = desc([2, 2])
    bad.s.numel = 5
    code, msg = call("rtc_relu", bad.ref, desc([2, 2]).ref)
    assert code == N.INVALID_ARGUMENT and "numel" in msg
    strided = desc([2, 3])
    st = (ctypes.c_size_t * 2)(1, 2)
    strided.s.strides = st
    code, msg = call("rtc_relu", strided.ref, desc([2, 3]).ref)
    assert code == N.UNSUPPORTED and "non-contiguous" in msg


def test_python_mirror_raises_valueerror_subclass():
    assert issubclass(N.RusttorchError, ValueError)


def test_sharded_stats_argument_checks_without_gpu():
    import ctypes as C
    L = N.lib()
    out = (C.c_double * 4)()
    r = L.rtc_sharded_stats(None, 0, out)          # nothing to reduce: the reference's
    assert not r.success and r.code == N.EMPTY_TENSOR   # empty-tensor error for max/min
    L.rtc_free_error_message(r.error_msg)
    assert out[0] == 0.0
    r = L.rtc_sharded_stats(None, 2, out)
    assert not r.success and r.code == N.INVALID_ARGUMENT
    L.rtc_free_error_message(r.error_msg)


def test_tensor_desc_keeps_its_tensor_alive():
    # A descriptor taken from a temporary tensor must not outlive its buffer:
    # Tensor.desc holds the tensor until the by-reference struct is dropped.
    import gc
    import weakref

    import rusttorch_b200 as rt
    t = rt.Tensor([2, 3], ptr=0x1000)       # borrowed address: nothing to free
    alive = weakref.ref(t)
    ref = t.desc
    del t
    gc.collect()
    assert alive() is not None
    s = ref._obj
    assert (s.ndim, s.numel, s.shape[0], s.shape[1], s.data) == (2, 6, 2, 3, 0x1000)
    del ref, s
    assert alive() is None                  # no cycle: freed without the collector


def test_nvtx_ranges_switched_on_by_the_environment():
    """RTC_NVTX=1 wraps every op in an NVTX range named after its entry point
    (read once per process, so this runs in a fresh one); calls behave the
    same with it on: a call that fails validation (no GPU needed) returns the
    same code and message as without it."""
    import sys
    code = (
        "from rusttorch_b200 import _native as N\n"
        "a = N.Desc(0, [2, 3], N.F32, 0)\n"
        "b = N.Desc(0, [3, 2], N.I32, 0)\n"
        "r = N.lib().rtc_add(a.ref, b.ref, a.ref)\n"
        "import ctypes\n"
        "print(r.code, ctypes.string_at(r.error_msg).decode())\n")
    env = dict(os.environ, RTC_NVTX="1")
    out = subprocess.run([sys.executable, "-c", code], env=env, cwd=str(ROOT),
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    a = N.Desc(0, [2, 3], N.F32, 0)
    b = N.Desc(0, [3, 2], N.I32, 0)
    r = N.lib().rtc_add(a.ref, b.ref, a.ref)
    want = f"{r.code} {ctypes.string_at(r.error_msg).decode()}"
    N.lib().rtc_free_error_message(r.error_msg)
    assert not r.success
    assert out.stdout.strip() == want


def test_peer_allreduce_argument_errors():
    """rtc_peer_allreduce_sum_f64 checks its arguments before touching a
    device: world beyond RTC_PEER_MAX_RANKS, a rank outside the world, a
    missing slot array, generation 0."""
    lib = N.lib()
    assert lib.rtc_peer_slot_bytes(8) == 2 * 8 * 16
    assert lib.rtc_peer_slot_bytes(0) == 0
    fake = ctypes.c_void_p(256)
    ptrs = (ctypes.c_void_p * 2)(256, 512)
    nulls = (ctypes.c_void_p * 2)(None, None)
    for world, rank, slots, gen in ((N.PEER_MAX_RANKS + 1, 0, ptrs, 1), (2, 2, ptrs, 1),
                                    (2, 0, nulls, 1), (2, 0, ptrs, 0)):
        with pytest.raises(N.RusttorchError) as e:
            N.check(lib.rtc_peer_allreduce_sum_f64(0, fake, slots, world, rank, gen, fake))
        assert e.value.code == N.INVALID_ARGUMENT
