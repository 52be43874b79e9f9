"""odf_flash_fwd_sm100_noalloc: the entry point for callers that cannot allocate
device memory (fixed-budget serving loops, plugins whose host owns the allocator,
foreign-language bindings without an allocator).  It keeps its work-item counter and
block-mask tile lists in a library-owned static device array instead of a caller
workspace.

Checked through the C ABI against odf_flash_fwd_sm100 (which uses a caller
workspace) on the same inputs, and on the greedy-counter path also against the
oracle, on two calls in a row so that a second call over the scratch left by the
first is covered too.  This file is collected last so a failure here never hides
the rest of the suite.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import make_qkv

pytestmark = pytest.mark.gpu

O_REL_L2 = 1e-2
O_MAX_ABS = 2e-2
LSE_MAX_ABS = 1e-3


def _lib():
    import odf_b200

    lib = odf_b200.load_library()
    lib.odf_flash_fwd_sm100_noalloc.argtypes = [C.POINTER(odf_b200.FwdParams), C.c_void_p]
    lib.odf_flash_fwd_sm100_noalloc.restype = C.c_int
    return lib


def _run(entry, q, k, v, mask, mask_block, causal, use_workspace, want_counter=False, alibi_slopes=None,
         softcap=0.0):
    """One call of `entry` on NaN-filled O/LSE (rows a call leaves out stay NaN).  With
    want_counter, also returns the work-item counter the workspace entry left in its workspace
    (0 when the launch used the fixed order, which never touches it)."""
    import odf_b200
    import torch

    B, Hq, M, D = q.shape
    o = torch.full((B, Hq, M, v.shape[3]), float("nan"), dtype=torch.float32, device="cuda")
    lse = torch.full((B, Hq, M), float("nan"), dtype=torch.float32, device="cuda")
    mask_t = torch.as_tensor(mask, dtype=torch.uint8).cuda().contiguous() if mask is not None else None
    p, keep = odf_b200.fill_params(q, k, v, o, lse, causal=causal, scale=1.0 / np.sqrt(D), block_mask=mask_t,
                                   mask_block=mask_block, alibi=alibi_slopes is not None,
                                   alibi_slopes_host=alibi_slopes, softcap=softcap, workspace=None, visits=None)
    ws = None
    if use_workspace:
        nbytes = _lib().odf_fwd_workspace_size(C.byref(p))
        if nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
            p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    rc = entry(C.byref(p), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, odf_b200.last_error()
    torch.cuda.synchronize()
    counter = int(ws[:8].cpu().numpy().view(np.uint64)[0]) if (want_counter and ws is not None) else None
    del keep, ws
    if want_counter:
        return o.cpu().numpy(), lse.cpu().numpy(), counter
    return o.cpu().numpy(), lse.cpu().numpy()


def _compare(o, lse, o_ref, lse_ref):
    diff = o.astype(np.float64) - o_ref.astype(np.float64)
    assert np.linalg.norm(diff) / max(np.linalg.norm(o_ref), 1e-30) <= O_REL_L2
    assert np.abs(diff).max() <= O_MAX_ABS
    fin = np.isfinite(lse_ref)
    assert np.array_equal(np.isfinite(lse), fin)
    assert np.abs(lse[fin] - lse_ref[fin]).max() <= LSE_MAX_ABS


@pytest.mark.parametrize("case", ["block_mask_causal", "block_mask_small_blocks", "causal_no_mask"])
def test_noalloc_matches_workspace_entry_two_calls(case):
    import torch

    import oracle

    lib = _lib()
    if case == "block_mask_causal":
        mask, mb, causal, n = oracle.sliding_window_prefix_mask(10, 3, 2), (128, 128), True, 1280
    elif case == "block_mask_small_blocks":
        rng = np.random.default_rng(3)
        mask, mb, causal, n = (rng.random((20, 15)) > 0.4).astype(np.uint8), (48, 64), False, 900
    else:
        mask, mb, causal, n = None, (128, 128), True, 700
    results = []
    for call in range(2):
        qn, kn, vn = make_qkv(40 + call, 2, 4, 2, n, n, 128)
        q, k, v = (torch.from_numpy(x).cuda().to(torch.bfloat16) for x in (qn, kn, vn))
        o_ref, lse_ref = _run(lib.odf_flash_fwd_sm100, q, k, v, mask, mb, causal, use_workspace=True)
        o, lse = _run(lib.odf_flash_fwd_sm100_noalloc, q, k, v, mask, mb, causal, use_workspace=False)
        _compare(o, lse, o_ref, lse_ref)
        results.append(o)
    assert not np.array_equal(results[0], results[1])  # the two calls really ran on different inputs


def test_noalloc_greedy_counter_path_two_calls_vs_oracle():
    """A problem long enough for the greedy, L2-blocked item order (plain score, d=128, K/V of
    16 (batch, kv-head) units = 64 MB, over the 32 MB block size), which hands out work through a
    counter: with the no-allocation entry that counter lives in the library's static scratch.
    Two calls in a row on NaN-filled outputs: a counter left uncleared by the first call would
    leave rows of the second unwritten.  Each call equals the workspace entry bit for bit (the
    item order does not change any item's arithmetic) and its causal prefix rows match the
    oracle.  N = 8192 (64 KV tiles) also selects the variant that skips the row-max pass."""
    import torch

    import oracle

    lib = _lib()
    B, H, N, D = 1, 16, 8192, 128
    n_items = B * H * (N // 256)  # work items: pairs of 128-row query tiles per (batch, head)
    for call in range(2):
        g = torch.Generator(device="cuda").manual_seed(70 + call)
        q, k, v = (torch.randn((B, H, N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
        o_ws, lse_ws, counter = _run(lib.odf_flash_fwd_sm100, q, k, v, None, (128, 128), True,
                                     use_workspace=True, want_counter=True)
        # the workspace entry chose the counter: every item taken, plus one failed take per CTA
        assert counter is not None and counter > n_items, f"counter {counter}: greedy order not used"
        o, lse = _run(lib.odf_flash_fwd_sm100_noalloc, q, k, v, None, (128, 128), True, use_workspace=False)
        assert np.isfinite(o).all() and np.isfinite(lse).all(), f"call {call}: rows left unwritten"
        assert np.array_equal(o, o_ws) and np.array_equal(lse, lse_ws), f"call {call}: differs from workspace entry"
        R, heads = 512, [0, 7, 15]
        qs, ks, vs = (t[:, heads, :R].float().cpu().numpy() for t in (q, k, v))
        o_ref, lse_ref = oracle.flash_fwd(qs, ks, vs, causal=True)
        _compare(o[:, heads, :R], lse[:, heads, :R], o_ref, lse_ref)


def test_noalloc_causal_alibi_far_bound_two_calls():
    """Causal ALiBi at d = 128 keeps its far-tile bound (tile norms, per-pair first KV tiles) and
    its greedy work-item counter in the scratch: two calls in a row on NaN-filled outputs, each
    bit for bit the workspace entry (same bound, same per-item arithmetic), with steep and flat
    slopes so that some pairs leave out far tiles and some none; soft-cap on the second call."""
    import torch

    lib = _lib()
    B, H, N, D = 1, 4, 2048, 128
    slopes = np.array([2.0, 0.5, 0.01, 0.0], dtype=np.float32)
    for call in range(2):
        g = torch.Generator(device="cuda").manual_seed(90 + call)
        q, k, v = (torch.randn((B, H, N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
        softcap = 30.0 if call else 0.0
        o_ws, lse_ws, counter = _run(lib.odf_flash_fwd_sm100, q, k, v, None, (128, 128), True, use_workspace=True,
                                     want_counter=True, alibi_slopes=slopes, softcap=softcap)
        assert counter is not None and counter > B * H * (N // 256), f"counter {counter}: greedy order not used"
        o, lse = _run(lib.odf_flash_fwd_sm100_noalloc, q, k, v, None, (128, 128), True, use_workspace=False,
                      alibi_slopes=slopes, softcap=softcap)
        assert np.isfinite(o).all() and np.isfinite(lse).all(), f"call {call}: rows left unwritten"
        assert np.array_equal(o, o_ws) and np.array_equal(lse, lse_ws), f"call {call}: differs from workspace entry"


def test_noalloc_rejects_lists_beyond_scratch():
    import odf_b200
    import torch

    lib = _lib()
    # 131072 x 131072 with a block mask needs 512 * 1024 * 4 bytes of lists > 1 MiB
    p = odf_b200.FwdParams()
    t = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    p.q = p.k = p.v = p.o = t.data_ptr()
    p.qkv_dtype, p.o_dtype = odf_b200.ODF_DTYPE_BF16, odf_b200.ODF_DTYPE_F32
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim, p.value_dim = 1, 1, 1, 131072, 131072, 64, 64
    p.scale = 0.125
    p.block_mask = t.data_ptr()
    p.mask_qbs = p.mask_kbs = 128
    p.mask_qblocks = p.mask_kblocks = 1
    rc = lib.odf_flash_fwd_sm100_noalloc(C.byref(p), None)
    assert rc == odf_b200.ODF_ERR_UNSUPPORTED
    assert "scratch" in odf_b200.last_error()
