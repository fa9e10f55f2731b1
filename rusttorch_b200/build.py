"""Build librusttorch_cuda.so (the sm_100a kernels and the C ABI) in-tree.

    python -m rusttorch_b200.build            # incremental
    python -m rusttorch_b200.build --force    # rebuild everything

nvcc compiles each csrc/*.cu for sm_100a only (-gencode arch=compute_100a,
code=sm_100a) with --fmad=false, so no a*b+c in device code is contracted
into an FMA unless the source asks for fma() explicitly (the reference's
arithmetic rounds every f32 operation once).  The shared library lands next
to this file so that it travels with the package.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "rusttorch_cuda"
LIB = PKG / "librusttorch_cuda.so"
HEADERS = [ROOT / "include" / "rusttorch_cuda.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--fmad=false",
    "-Xcompiler",
    "-fPIC,-O2,-Wall",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def cuda_lib_dir() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(cuda) / "lib64")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool, ptxas_v: bool) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if ptxas_v or verbose:
        sys.stderr.write(res.stderr)


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    """Compile every csrc/*.cu and link librusttorch_cuda.so; returns its path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + HEADERS
    objs = []
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_v or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            list(ex.map(lambda j: _compile(j[0], j[1], verbose, ptxas_v), jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs),
               "-L", cuda_lib_dir(), "-lcudart", "-Xlinker", "-rpath," + cuda_lib_dir()]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v))


if __name__ == "__main__":
    main()
