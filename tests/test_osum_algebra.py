"""The losses' ordered-sum algebra (rusttorch_b200/csrc/rt_osum.cuh) on the CPU.

The per-binade moves, run composition and application are host-callable, so
tests/osum_algebra_check.cu builds against the header with nvcc and checks
them against plain sequential f32 adds (and an emulation of the kernels'
pipeline against ndarray's eight-chain fold and a one-chain fold), with no
GPU.  The GPU kernels themselves are checked in tests/test_ordered_sum.py.
"""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(cuda) / "bin" / "nvcc"
    return str(p) if p.exists() else shutil.which("nvcc")


@pytest.mark.skipif(_nvcc() is None, reason="nvcc not found")
def test_osum_algebra_on_host(tmp_path):
    exe = tmp_path / "osum_algebra_check"
    build = subprocess.run(
        [_nvcc(), "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
         "-I", str(ROOT / "rusttorch_b200" / "csrc"), "-o", str(exe),
         str(ROOT / "tests" / "osum_algebra_check.cu")],
        capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0 and "ALL OK" in run.stdout, run.stdout + run.stderr
