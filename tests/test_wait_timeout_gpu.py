"""Bounded in-kernel waits: a wait that runs out ends the launch with a status, not a hang.

Failure drill through the C ABI's test hook odf_debug_set_wait: the wait limit is lowered
to 20 ms and CTA 0's producer warp leaves out one K/V tile load, so the MMA warp's wait for
that ring slot can never complete.  The launch must then finish on its own (well inside a
second, against the 2 s default limit), the device status word must read
ODF_ERR_DEVICE_TIMEOUT, and the same process must run a normal launch afterwards that
matches the oracle -- the copies and MMAs in flight were drained and the tensor memory
freed, so the context stays usable.  Nothing here faults or traps the GPU: the failure is a
load that is never issued, and every wait in the kernel is bounded.
"""
from __future__ import annotations

import ctypes as C
import time

import numpy as np
import pytest

from conftest import make_qkv

pytestmark = pytest.mark.gpu

LIMIT_NS = 20_000_000  # 20 ms


def _hook():
    import odf_b200

    lib = odf_b200.load_library()
    lib.odf_debug_set_wait.argtypes = [C.c_uint64, C.c_int32]
    lib.odf_debug_set_wait.restype = C.c_int
    return lib


@pytest.mark.parametrize("case", ["d128_first_load", "d128_mid_item", "d64_mid_item", "d128_greedy_order"])
def test_wait_runs_out_and_context_recovers(case):
    import odf_b200
    import oracle
    import torch

    lib = _hook()
    assert odf_b200.device_status(clear=True) == 0
    if case == "d128_first_load":  # nothing issued by the MMA warp yet
        B, H, N, D, stall = 1, 2, 2048, 128, 0
    elif case == "d128_mid_item":  # S and P.V MMAs of the first KV tiles in flight
        B, H, N, D, stall = 1, 2, 2048, 128, 5
    elif case == "d64_mid_item":   # the separate-P layout (d = 64) with its extra barriers
        B, H, N, D, stall = 1, 2, 2048, 64, 5
    else:                          # items handed out through the workspace counter and item queue
        B, H, N, D, stall = 1, 16, 8192, 128, 3
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn((B, H, N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    torch.cuda.synchronize()
    assert lib.odf_debug_set_wait(LIMIT_NS, stall) == 0
    try:
        t0 = time.perf_counter()
        odf_b200.flash_fwd(q, k, v, causal=True)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        assert lib.odf_debug_set_wait(0, -1) == 0
    assert odf_b200.device_status(clear=True) == odf_b200.ODF_ERR_DEVICE_TIMEOUT
    assert elapsed < 1.0, f"the stalled launch took {elapsed:.3f} s (limit {LIMIT_NS / 1e6} ms)"

    # the same process, the same context: a normal launch is correct and sets no status
    qn, kn, vn = make_qkv(12, 1, 2, 2, 640, 640, D)
    dev = [torch.from_numpy(x).cuda().to(torch.bfloat16) for x in (qn, kn, vn)]
    o, lse = odf_b200.flash_fwd(*dev, causal=True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.flash_fwd(qn, kn, vn, causal=True)
    o = o.cpu().numpy()
    assert np.linalg.norm(o - o_ref) / np.linalg.norm(o_ref) <= 1e-2
    assert np.abs(o - o_ref).max() <= 2e-2
    assert np.abs(lse.cpu().numpy() - lse_ref).max() <= 1e-3
    assert odf_b200.device_status(clear=True) == 0


def test_debug_hook_is_per_thread_and_off_by_default():
    """The hook only affects the thread that set it: another thread's launch runs normally."""
    import threading

    import odf_b200
    import torch

    lib = _hook()
    assert lib.odf_debug_set_wait(LIMIT_NS, 0) == 0
    try:
        q, k, v = make_qkv(13, 1, 2, 2, 512, 512, 128)
        out = {}

        def worker():
            torch.cuda.set_device(0)
            dev = [torch.from_numpy(x).cuda().to(torch.bfloat16) for x in (q, k, v)]
            o, _ = odf_b200.flash_fwd(*dev, causal=True)
            torch.cuda.synchronize()
            out["o"] = o.cpu().numpy()

        t = threading.Thread(target=worker)
        t.start()
        t.join()
    finally:
        assert lib.odf_debug_set_wait(0, -1) == 0
    assert odf_b200.device_status(clear=True) == 0
    assert np.isfinite(out["o"]).all()
