"""rtc_sum_device_noalloc against rtc_sum_device (GPU).

The no-allocation variant exists for callers that may not allocate GPU
memory themselves (their memory is reserved by another allocator, or their
policy or latency budget forbids it); it keeps its scratch in a fixed array
inside the library.  Both entry points run the same two kernels with the
same number of partial sums, so the results must be equal bit for bit, on
consecutive calls: a large input first, then a smaller one that uses fewer
partials, so partials the first call left behind in the shared array would
show if the second call read them.

This file is collected last on purpose, and it must pass both alone in a
fresh process and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

from rusttorch_b200 import _native as N
from tests import _oracle as O

pytestmark = pytest.mark.gpu


def _device_sum(fn, t, out):
    N.check(fn(t.desc, ctypes.c_void_p(out.ptr)))
    N.check(N.lib().rtc_synchronize())
    v = np.empty(1, np.float64)
    N.check(N.lib().rtc_memcpy_d2h(t.device, v.ctypes.data_as(ctypes.c_void_p),
                                   ctypes.c_void_p(out.ptr), 8))
    return float(v[0])


def test_noalloc_sum_matches_allocating_sum_twice():
    import rusttorch_b200 as rt

    lib = N.lib()
    out = rt.Tensor([2])          # 8 bytes of device memory for the f64 result
    # two calls in a row: 2^26 elements (1184 partials on a B200), then
    # 1_000_003 (62 partials)
    for seed, n in ((2, 1 << 26), (9, 1_000_003)):
        x = O.normal(n, seed)
        t = rt.Tensor.from_numpy(x)
        want = _device_sum(lib.rtc_sum_device, t, out)
        got = _device_sum(lib.rtc_sum_device_noalloc, t, out)
        assert got == want, (n, got, want)
        tol = 1e-6 * float(np.abs(x.astype(np.float64)).sum())
        assert abs(got - O.sum(x)) <= tol, (n, got, O.sum(x))


def test_noalloc_sum_of_empty_is_zero():
    import rusttorch_b200 as rt

    out = rt.Tensor([2])
    empty = N.Desc(0, [0], N.F32, 0)
    N.check(N.lib().rtc_sum_device_noalloc(empty.ref, ctypes.c_void_p(out.ptr)))
    N.check(N.lib().rtc_synchronize())
    v = np.ones(1, np.float64)
    N.check(N.lib().rtc_memcpy_d2h(0, v.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(out.ptr), 8))
    assert v[0] == 0.0
