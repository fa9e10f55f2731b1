"""The tolerance math mode against the reference's formulas (CPU).

rusttorch_b200/csrc/rt_fastmath.cuh and the *Tol rules of rt_ops.cuh
compute every step as one IEEE operation, so their host build gives the
device's bits (tests/test_tolerance_gpu.py checks that on the GPU).  Here
that host build is compared with the reference's formula over glibc for
every input of a strided sweep of all 2^32 float bit patterns (RT_EXHAUSTIVE=1:
all of them, about a minute per op on 16 cores): no input may miss
north_star's tolerance, 1e-6 relative error or 4 ulp, and the largest
relative error is held to the figure the library documents.
"""
import ctypes
import os
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

from rusttorch_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "native" / "fastmath_check.cpp"
DEPS = [SRC] + [ROOT / "rusttorch_b200" / "csrc" / h
                for h in ("rt_fastmath.cuh", "rt_libm.cuh", "rt_ops.cuh")]
LIB = ROOT / "_build" / "fastmath_check.so"

OPS = {"sigmoid": 0, "swish": 1, "tanh": 2, "softplus": 3, "mish": 4, "gelu": 5, "exp": 6,
       "log": 7}
# Largest relative error over all 2^32 inputs (normal results), measured
# exhaustively; the strided sweep must stay within it.
MAX_REL = {"sigmoid": 2.7e-7, "swish": 3.3e-7, "tanh": 2.4e-7, "softplus": 1.2e-7,
           "mish": 4.8e-7, "gelu": 5.8e-7, "exp": 1.2e-7, "log": 1.2e-7}


def load_fastmath_lib():
    LIB.parent.mkdir(parents=True, exist_ok=True)
    newest = max(p.stat().st_mtime for p in DEPS)
    if not LIB.exists() or newest > LIB.stat().st_mtime:
        subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
                        "-shared", "-pthread", "-o", str(LIB), str(SRC), "-lm"], check=True)
    lib = ctypes.CDLL(str(LIB))
    lib.fm_scan.restype = ctypes.c_uint64
    lib.fm_scan.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                            ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                            ctypes.POINTER(ctypes.c_uint32)]
    for fn in (lib.fm_eval, lib.fm_ref):
        fn.restype = None
        fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64]
    return lib


@pytest.fixture(scope="module")
def fm():
    return load_fastmath_lib()


def f32(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


@pytest.mark.parametrize("op", list(OPS))
def test_within_tolerance_on_a_sweep_of_all_floats(fm, op):
    stride = 1 if os.environ.get("RT_EXHAUSTIVE") == "1" else 211
    stats = (ctypes.c_double * 2)()
    worst = (ctypes.c_uint32 * 2)()
    n = fm.fm_scan(OPS[op], 0, 1 << 32, stride, os.cpu_count() or 1, stats, worst)
    assert n == 0, f"{op}: {n} inputs miss 1e-6 rel / 4 ulp; first x={f32(worst[0])!r}"
    assert stats[1] <= MAX_REL[op], (op, stats[1], f32(worst[1]))


# Inputs at the rules' branch points and thresholds: expf's overflow
# (+-88.7228...), softplus/mish's x > 20, tanh's |x| = 0.55 and 9.5, GELU's
# exact range (-1.4 > z >= -9.1, i.e. x near -1.58 and -5.25), exp's clamps.
EDGES = [0.0, -0.0, 1e-45, -1e-45, 1.17549435e-38, -1.17549435e-38, 0.5, -0.5, 0.55, -0.55,
         0.5499999, 9.5, -9.5, 9.02, -9.02, 20.0, 20.000002, 19.999998, -20.0, 88.72283172607422,
         88.72283935546875, -88.72283172607422, -88.72283935546875, -88.7228, -87.33, -103.97,
         -104.0, -104.00001, 89.0, 89.00001, -1.5, -1.58, -1.6, -5.25, -5.3, -16.6, -17.0, 1e30,
         -1e30, 3.4028235e38, -3.4028235e38, np.inf, -np.inf]


@pytest.mark.parametrize("op", ["sigmoid", "swish", "tanh", "softplus", "mish", "gelu", "exp"])
def test_edges(fm, op):
    x = np.array(EDGES, dtype=np.float32)
    x = np.concatenate([x, np.nextafter(x, np.float32(np.inf)), np.nextafter(x, -np.float32(np.inf))])
    got, want = np.empty_like(x), np.empty_like(x)
    fm.fm_eval(OPS[op], x.ctypes.data, got.ctypes.data, x.size)
    fm.fm_ref(OPS[op], x.ctypes.data, want.ctypes.data, x.size)
    both_nan = np.isnan(got) & np.isnan(want)
    assert not (np.isnan(got) ^ np.isnan(want)).any(), (op, x[np.isnan(got) ^ np.isnan(want)])
    g, w = got[~both_nan], want[~both_nan]
    ulps = np.abs(ordered(g) - ordered(w))
    with np.errstate(invalid="ignore", divide="ignore"):
        rel = np.where(g == w, 0.0, np.abs(g.astype(np.float64) - w) / np.abs(w.astype(np.float64)))
    bad = (ulps > 4) & (rel > 1e-6)
    assert not bad.any(), (op, x[~both_nan][bad], g[bad], w[bad])


def ordered(a):
    """float32 bit patterns mapped to integers in the floats' order (+0 and
    -0 both to 0), so that a difference counts ulps."""
    i = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.int64)
    return np.where(i < 0x80000000, i, 0x80000000 - i)


def test_zero_results_where_the_reference_overflows(fm):
    """expf(88.72283935546875) is +inf in glibc, so the reference's sigmoid
    is exactly +0 and swish exactly -0 at and below -88.72283935546875."""
    x = np.array([-88.72283935546875, -90.0, -1e10, -np.inf], dtype=np.float32)
    out = np.empty_like(x)
    fm.fm_eval(OPS["sigmoid"], x.ctypes.data, out.ctypes.data, x.size)
    assert (out.view(np.uint32) == 0).all()
    fm.fm_eval(OPS["swish"], x[:3].ctypes.data, out.ctypes.data, 3)
    assert (out[:3].view(np.uint32) == 0x80000000).all()


def test_math_mode_switch_without_a_gpu():
    lib = N.lib()
    before = lib.rtc_get_math_mode()
    try:
        N.check(lib.rtc_set_math_mode(N.MATH_EXACT))
        assert lib.rtc_get_math_mode() == N.MATH_EXACT
        N.check(lib.rtc_set_math_mode(N.MATH_TOLERANCE))
        assert lib.rtc_get_math_mode() == N.MATH_TOLERANCE
        with pytest.raises(N.RusttorchError) as e:
            N.check(lib.rtc_set_math_mode(7))
        assert e.value.code == N.INVALID_ARGUMENT
    finally:
        N.check(lib.rtc_set_math_mode(before))
