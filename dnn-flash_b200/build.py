"""Build step for the sm_100a library (lib/libodf_sm100.so).

Plain nvcc, in-tree, so the shared object travels with the source tree:
    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -shared ...
The CUDA runtime is linked statically; the driver API (cuTensorMapEncodeTiled)
is fetched at run time through cudaGetDriverEntryPoint, so no -lcuda.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
LIB = PACKAGE_DIR / "lib" / "libodf_sm100.so"
# The same sources with the in-kernel invariant checks compiled in (-DODF_CHECKED): test
# infrastructure (tests/test_checked_build_gpu.py), never loaded by the package itself.
CHECKED_LIB = PACKAGE_DIR / "lib" / "libodf_sm100_checked.so"
SOURCES = [CSRC / "flash_fwd_sm100.cu", CSRC / "odf_capi.cu"]
CXX_API_SOURCES = [CSRC / "onednn_flash_api.cpp", CSRC / "planner.cpp"]
DEPS = SOURCES + CXX_API_SOURCES + [CSRC / "sm100_ptx.cuh", CSRC / "softmax_math.cuh", CSRC / "odf_internal.h"] + sorted(
    (ROOT / "include").rglob("*.h*"))
# Test-only device wrappers of the softmax arithmetic helpers (error-bound tests).
MATH_CHECK_SRC = ROOT / "tests" / "cuda" / "math_check.cu"
MATH_CHECK_LIB = ROOT / "tests" / "cuda" / "lib" / "libodf_math_check.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xlinker", "-Bsymbolic",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def up_to_date(lib: Path = LIB) -> bool:
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPS if p.exists())


def build_library(force: bool = False, verbose: bool = False, checked: bool = False) -> Path:
    lib = CHECKED_LIB if checked else LIB
    if not force and up_to_date(lib):
        return lib
    lib.parent.mkdir(parents=True, exist_ok=True)
    srcs = [str(s) for s in SOURCES + CXX_API_SOURCES if s.exists()]
    cmd = [nvcc(), *NVCC_FLAGS, *(["-DODF_CHECKED"] if checked else []), f"-I{ROOT / 'include'}", f"-I{CSRC}",
           "-shared", "-o", str(lib) + ".tmp", *srcs]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(lib) + ".tmp", lib)
    return lib


def build_math_check(force: bool = False, verbose: bool = False) -> Path:
    """tests/cuda/lib/libodf_math_check.so (test infrastructure, not part of the library)."""
    deps = [MATH_CHECK_SRC, CSRC / "softmax_math.cuh", CSRC / "sm100_ptx.cuh", CSRC / "odf_internal.h"]
    if not force and MATH_CHECK_LIB.exists() and all(
            p.stat().st_mtime <= MATH_CHECK_LIB.stat().st_mtime for p in deps):
        return MATH_CHECK_LIB
    MATH_CHECK_LIB.parent.mkdir(parents=True, exist_ok=True)
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{ROOT / 'include'}", f"-I{CSRC}", "-shared", "-o", str(MATH_CHECK_LIB) + ".tmp",
           str(MATH_CHECK_SRC)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(MATH_CHECK_LIB) + ".tmp", MATH_CHECK_LIB)
    return MATH_CHECK_LIB


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose=True)
    build_library(force="--force" in sys.argv, verbose=True, checked=True)
    build_math_check(force="--force" in sys.argv, verbose=True)
    print(LIB)
