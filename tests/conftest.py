"""Test configuration.

`-m gpu` tests need a B200 and call the CUDA path through the C ABI; every
other test runs on the CPU (oracle vs golden vectors, host logic, ABI symbol
and validation checks that return before any device work, gloo ranks).
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the CUDA path")


def _build_oracle():
    lib = ROOT / "oracle" / "liboracle.so"
    src = [ROOT / "oracle" / "rt_oracle.c", ROOT / "oracle" / "rt_oracle.h"]
    if not lib.exists() or any(s.stat().st_mtime > lib.stat().st_mtime for s in src):
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)


def _build_native():
    from rusttorch_b200 import build as b
    b.build()


@pytest.fixture(scope="session", autouse=True)
def _built():
    _build_oracle()
    # The CUDA library cross-compiles without a GPU; build it if stale.
    if os.environ.get("RT_SKIP_NATIVE_BUILD") != "1":
        try:
            _build_native()
        except Exception as e:  # nvcc missing on a box that only runs the GPU tests
            if not (ROOT / "rusttorch_b200" / "librusttorch_cuda.so").exists():
                raise
            print(f"warning: rebuild skipped: {e}", file=sys.stderr)
    yield


@pytest.fixture(scope="module")
def exact_math():
    """Runs a module's tests in the exact math mode (glibc's expf/tanhf
    reproduced bit for bit) and restores the mode afterwards; the library's
    default is the tolerance mode."""
    from rusttorch_b200 import _native as N
    lib = N.lib()
    before = lib.rtc_get_math_mode()
    N.check(lib.rtc_set_math_mode(N.MATH_EXACT))
    yield
    N.check(lib.rtc_set_math_mode(before))
