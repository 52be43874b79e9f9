"""Division by a launch-invariant divisor (odf::make_fastdiv / odf::fast_div in
dnn-flash_b200/csrc/odf_internal.h), which the kernels use to decode work items in 32-bit
arithmetic: every quotient must equal x // d exactly.  This file checks the host build on the CPU
over the divisors the decode meets (heads, kv-head groups, items per block and per query-tile
pair) and awkward ones (1, powers of two and their neighbours, 2^31 - 1, 2^32 - 1), against
random and edge dividends; tests/test_math_check_gpu.py checks the device build the same way.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

LIB = Path(__file__).resolve().parent / "cuda" / "lib" / "libodf_math_check.so"

DIVISORS = sorted({1, 2, 3, 5, 6, 7, 8, 9, 12, 16, 24, 31, 32, 33, 48, 64, 96, 100, 127, 128, 129, 255, 256, 257,
                   1000, 1023, 1024, 1025, 2048, 4095, 65535, 65536, 65537, 2 ** 24 - 1, 2 ** 24 + 1, 2 ** 31 - 1,
                   2 ** 31, 2 ** 31 + 1, 2 ** 32 - 1, 1 * 64 * 128, 8 * 16 * 8, 2 * 8 * 128, 3 * 8 * 256, 100003})


def dividends(d: int, rng) -> np.ndarray:
    edge = [0, 1, 2, d - 1, d, d + 1, 2 * d - 1, 2 * d, 2 ** 31 - 1, 2 ** 31, 2 ** 32 - 1, 2 ** 32 - 2]
    mult = [(2 ** 32 - 1) // d * d, (2 ** 32 - 1) // d * d - 1]
    x = np.concatenate([np.array([v for v in edge + mult if 0 <= v < 2 ** 32], dtype=np.uint64),
                        rng.integers(0, 2 ** 32, size=20000, dtype=np.uint64),
                        rng.integers(0, 1 << 20, size=5000, dtype=np.uint64)])
    return x.astype(np.uint32)


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        pytest.fail(f"{LIB} is missing: build it with __graft_entry__.build()")
    lib = C.CDLL(str(LIB))
    lib.odf_math_check_fastdiv_host.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_int64]
    lib.odf_math_check_fastdiv_host.restype = None
    return lib


@pytest.mark.parametrize("d", DIVISORS)
def test_fastdiv_host_exact(lib, d):
    rng = np.random.default_rng(d)
    x = dividends(d, rng)
    q = np.zeros_like(x)
    lib.odf_math_check_fastdiv_host(d, x.ctypes.data, q.ctypes.data, x.size)
    np.testing.assert_array_equal(q, (x.astype(np.uint64) // d).astype(np.uint32))
