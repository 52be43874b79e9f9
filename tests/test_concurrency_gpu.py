"""Concurrent use of the C ABI, as the reference's contract allows for its own entry points.

The reference keeps one workspace per host thread (thread_local in
src/onednn_flash/batched_attention.cpp:37) so several threads may run attention at
once.  The GPU library's counterparts:
  * odf_flash_fwd_host keeps its device buffers and streams per host thread, so two threads
    may call it at the same time;
  * odf_flash_fwd_sm100 is asynchronous on the caller's stream and keeps no state between
    calls apart from the caller's workspace, so launches on two streams with separate
    workspaces may overlap on the GPU.
Each concurrent result must equal the serial result bit for bit (every work item's
arithmetic is fixed, whichever CTA or stream runs it).
"""
from __future__ import annotations

import ctypes as C
import math
import threading

import numpy as np
import pytest

from conftest import make_qkv

pytestmark = pytest.mark.gpu


def _host_call(q, k, v, kw):
    import odf_b200

    lse = np.empty(q.shape[:3], dtype=np.float32)
    o, _ = odf_b200.flash_fwd_host(q, k, v, lse_out=lse, **kw)
    return o, lse


def test_two_host_threads_on_the_host_entry():
    """Two threads call odf_flash_fwd_host at once, three times each, on different problems
    (a plain causal GQA one and an ALiBi + block-mask one); every result equals the serial one."""
    import oracle

    problems = [
        (make_qkv(81, 2, 8, 2, 1500, 1500, 128), dict(causal=True)),
        (make_qkv(82, 1, 6, 6, 1024, 1024, 64),
         dict(causal=True, alibi=True, block_mask=oracle.sliding_window_prefix_mask(8, 3, 2),
              mask_block=(128, 128))),
    ]
    serial = [_host_call(*qkv, kw) for qkv, kw in problems]
    results = [[], []]
    errors = []
    barrier = threading.Barrier(2)

    def worker(i):
        try:
            import torch

            torch.cuda.set_device(0)
            barrier.wait()
            for _ in range(3):
                results[i].append(_host_call(*problems[i][0], problems[i][1]))
        except Exception as exc:  # reported below, in the main thread
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for i in range(2):
        assert len(results[i]) == 3
        for o, lse in results[i]:
            assert np.array_equal(o, serial[i][0]), f"thread {i}: O differs from the serial call"
            assert np.array_equal(lse, serial[i][1]), f"thread {i}: LSE differs from the serial call"


def test_two_streams_with_separate_workspaces():
    """Launches of odf_flash_fwd_sm100 on two streams, each with its own workspace, overlap on
    the GPU: stream 1 runs a long plain problem that hands out work through the counter in its
    workspace, stream 2 a block-mask problem whose tile lists live in its workspace.  Each
    stream's results equal the serial launches bit for bit."""
    import odf_b200
    import oracle
    import torch

    lib = odf_b200.load_library()
    g = torch.Generator(device="cuda").manual_seed(90)
    qa, ka, va = (torch.randn((1, 16, 8192, 128), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    qb, kb, vb = (torch.randn((2, 4, 2048, 64), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    mask = torch.as_tensor(oracle.sliding_window_prefix_mask(16, 4, 2)).cuda()

    def prepare(q, k, v, causal, block_mask):
        o = torch.empty(q.shape, dtype=torch.float32, device="cuda")
        lse = torch.empty(q.shape[:3], dtype=torch.float32, device="cuda")
        p, keep = odf_b200.fill_params(q, k, v, o, lse, causal=causal, scale=1.0 / math.sqrt(q.shape[3]),
                                       block_mask=block_mask, mask_block=(128, 128), alibi=False,
                                       alibi_slopes_host=None, softcap=0.0, workspace=None, visits=None)
        ws = torch.zeros(lib.odf_fwd_workspace_size(C.byref(p)), dtype=torch.uint8, device="cuda")
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        return p, (o, lse, ws, keep)

    def launch(p, stream):
        assert lib.odf_flash_fwd_sm100(C.byref(p), C.c_void_p(stream.cuda_stream)) == 0, odf_b200.last_error()

    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    pa, ra = prepare(qa, ka, va, True, None)
    pb, rb = prepare(qb, kb, vb, False, mask)
    torch.cuda.synchronize()
    launch(pa, s1)
    torch.cuda.synchronize()
    launch(pb, s2)
    torch.cuda.synchronize()
    serial = [(ra[0].clone(), ra[1].clone()), (rb[0].clone(), rb[1].clone())]
    for _ in range(3):
        ra[0].fill_(float("nan"))
        rb[0].fill_(float("nan"))
        torch.cuda.synchronize()
        launch(pa, s1)
        launch(pb, s2)
        torch.cuda.synchronize()
        assert torch.equal(ra[0], serial[0][0]) and torch.equal(ra[1], serial[0][1]), "stream 1 differs"
        assert torch.equal(rb[0], serial[1][0]) and torch.equal(rb[1], serial[1][1]), "stream 2 differs"
    # the block-mask problem also against the oracle, so the serial reference is itself checked
    o_ref, lse_ref = oracle.flash_fwd(qb.float().cpu().numpy(), kb.float().cpu().numpy(), vb.float().cpu().numpy(),
                                      mask=oracle.sliding_window_prefix_mask(16, 4, 2), mask_block=(128, 128))
    o = serial[1][0].cpu().numpy()
    assert np.linalg.norm(o - o_ref) / np.linalg.norm(o_ref) <= 1e-2
    assert odf_b200.device_status(clear=True) == 0
