"""Error bounds of the softmax warps' own arithmetic, run on the GPU, checked against exact
values computed on the host in float64.

* exp2_poly2 (dnn-flash_b200/csrc/softmax_math.cuh): 2^x on the FMA pipe from a degree-3
  polynomial fitted here (minimax relative error with p(0) = 1), used for one exponential pair
  in eight at d = 64.  Bound: relative error <= 1.02e-4 wherever 2^x is a normal float
  (x >= -126); exactly +0 at x <= -127 and at -inf; below 2^-126 in between.  The hardware
  ex2.approx on the same inputs is reported beside it for scale.
* tanh2: the soft-cap softcap * tanh(s / softcap) from the MUFU tanh.approx.f32.  PTX documents
  only a 2^-11 relative bound for that instruction; on sm_100 it measures 7.8e-6 absolute at
  worst, and the attention parity tolerances (LSE 1e-3 with soft-caps down to 5) rely on that,
  so this test pins an absolute error <= 1e-5 * softcap over |s| up to 40 * softcap: a GPU or
  driver whose tanh.approx is less accurate fails here, before the parity tests.

The device side is tests/cuda/math_check.cu, a test-only library around the same header the
kernel includes.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent / "cuda" / "lib" / "libodf_math_check.so"
EXP2_REL_BOUND = 1.02e-4
SOFTCAP_ABS_BOUND = 1e-5  # times softcap


def _lib():
    if not LIB.exists():
        raise ImportError(f"{LIB} is missing: build it with __graft_entry__.build()")
    lib = C.CDLL(str(LIB))
    lib.odf_math_check_exp2.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]
    lib.odf_math_check_softcap.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_float]
    lib.odf_math_check_fastdiv.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_int64]
    return lib


def test_exp2_poly2_error_bound():
    import torch

    lib = _lib()
    dense = np.linspace(-130.0, 8.0, 1 << 21, dtype=np.float32)
    rng = np.random.default_rng(5)
    near_int = (np.arange(-127, 9)[:, None] + np.float32([-0.5, -0.25, -1e-6, 0.0, 1e-6, 0.25, 0.4999])[None, :])
    special = np.float32([-np.inf, -127.0, -126.5, -126.0, -1e-30, 0.0, 1e-30, 8.0])
    x = np.concatenate([dense, rng.uniform(-127.0, 8.0, 1 << 20).astype(np.float32),
                        near_int.ravel().astype(np.float32), special]).astype(np.float32)
    if x.size % 2:
        x = np.append(x, np.float32(0.0))
    xd = torch.from_numpy(x).cuda()
    yp = torch.empty_like(xd)
    ym = torch.empty_like(xd)
    assert lib.odf_math_check_exp2(xd.data_ptr(), yp.data_ptr(), ym.data_ptr(), x.size) == 0
    poly = yp.cpu().numpy().astype(np.float64)
    mufu = ym.cpu().numpy().astype(np.float64)
    exact = np.exp2(x.astype(np.float64))
    normal = x >= -126.0
    rel = np.abs(poly[normal] - exact[normal]) / exact[normal]
    rel_mufu = np.abs(mufu[normal] - exact[normal]) / exact[normal]
    print(f"exp2_poly2 max rel {rel.max():.3e} (x = {x[normal][rel.argmax()]}); ex2.approx max rel {rel_mufu.max():.3e}")
    assert rel.max() <= EXP2_REL_BOUND
    assert np.all(poly[x <= -127.0] == 0.0) and not np.signbit(poly[x <= -127.0]).any()
    between = (x > -127.0) & (x < -126.0)
    assert np.all((poly[between] >= 0.0) & (poly[between] < 2.0 ** -126))


@pytest.mark.parametrize("softcap", [5.0, 30.0, 50.0])
def test_softcap_tanh_error_bound(softcap):
    import torch

    lib = _lib()
    rng = np.random.default_rng(int(softcap))
    s = np.concatenate([np.linspace(-40 * softcap, 40 * softcap, 1 << 20),
                        rng.standard_normal(1 << 20) * softcap,
                        np.float32([0.0, -0.0, 1e-30, -1e-30, softcap, -softcap])]).astype(np.float32)
    if s.size % 2:
        s = np.append(s, np.float32(0.0))
    sd = torch.from_numpy(s).cuda()
    y = torch.empty_like(sd)
    assert lib.odf_math_check_softcap(sd.data_ptr(), y.data_ptr(), s.size, softcap) == 0
    got = y.cpu().numpy().astype(np.float64)
    exact = softcap * np.tanh(s.astype(np.float64) / softcap)
    err = np.abs(got - exact).max()
    print(f"softcap {softcap}: max abs error {err:.3e} ({err / softcap:.2e} x softcap)")
    assert err <= SOFTCAP_ABS_BOUND * softcap
    big = np.abs(exact) > 1e-5 * softcap
    assert np.all(np.sign(got[big]) == np.sign(exact[big]))


def test_fastdiv_device_exact():
    """The device build of the item decode's division (multiply-high instruction) equals x // d
    for the divisors and dividends of tests/test_fastdiv.py."""
    import torch

    from test_fastdiv import DIVISORS, dividends

    lib = _lib()
    rng = np.random.default_rng(7)
    for d in DIVISORS:
        x = dividends(d, rng)
        xd = torch.from_numpy(x.view(np.int32)).cuda()
        qd = torch.empty_like(xd)
        assert lib.odf_math_check_fastdiv(d, xd.data_ptr(), qd.data_ptr(), x.size) == 0
        q = qd.cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(q, (x.astype(np.uint64) // d).astype(np.uint32), err_msg=f"d={d}")
