"""Runs the checked build (libodf_sm100_checked.so: the library compiled with its in-kernel
invariant checks) over a set of problems that reach every scheduling and score-mod path, and
prints one JSON line per case: the status word, the failed-check bits and the parity against the
oracle.  Started as its own process by tests/test_checked_build_gpu.py, so that the checked
library is the only copy of the library in that process.
"""
from __future__ import annotations

import ctypes as C
import json
import sys
import zlib
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "dnn-flash_b200"))
sys.path.insert(0, str(ROOT / "tests"))
sys.path.insert(0, str(ROOT))

import odf_b200  # noqa: E402

odf_b200.LIB_PATH = ROOT / "dnn-flash_b200" / "lib" / "libodf_sm100_checked.so"

from conftest import make_qkv  # noqa: E402
import oracle  # noqa: E402
import torch  # noqa: E402


def parity(o, lse, o_ref, lse_ref):
    diff = o.astype(np.float64) - o_ref.astype(np.float64)
    rel = float(np.linalg.norm(diff) / max(np.linalg.norm(o_ref.astype(np.float64)), 1e-30))
    fin = np.isfinite(lse_ref)
    lse_err = float(np.abs(lse[fin] - lse_ref[fin]).max()) if fin.any() else 0.0
    return {"o_rel_l2": rel, "o_max_abs": float(np.abs(diff).max()), "lse_max_abs": lse_err,
            "lse_inf_pattern": bool(np.array_equal(np.isfinite(lse), fin))}


def run_case(name, B, Hq, Hkv, M, N, D, entry="device", prefix=None, in_scale=1.0, **kw):
    q, k, v = make_qkv(zlib.crc32(name.encode()) % 100000, B, Hq, Hkv, M, N, D, scale=in_scale)
    slopes = kw.pop("alibi_slopes", None)
    alibi = kw.pop("alibi", False) or slopes is not None
    bias = kw.pop("bias", None)
    if entry == "device":
        dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(torch.bfloat16)
        o_t, lse_t = odf_b200.flash_fwd(dev(q), dev(k), dev(v), alibi=alibi, alibi_slopes=slopes,
                                        bias=torch.from_numpy(bias).cuda() if bias is not None else None, **kw)
        torch.cuda.synchronize()
        o, lse = o_t.float().cpu().numpy(), lse_t.cpu().numpy()
    else:
        lse = np.empty((B, Hq, M), dtype=np.float32)
        o, _ = odf_b200.flash_fwd_host(q, k, v, alibi=alibi, alibi_slopes=slopes, bias=bias, lse_out=lse, **kw)
    lib = odf_b200.load_library()
    bits = C.c_uint32(0)
    rc = lib.odf_debug_check_bits(C.byref(bits))
    status = odf_b200.device_status()
    okw = dict(causal=kw.get("causal", False), softcap=kw.get("softcap", 0.0), mask=kw.get("block_mask"),
               mask_block=kw.get("mask_block", (128, 128)), bias=bias,
               alibi_slopes=(slopes if slopes is not None else oracle.alibi_slopes(Hq)) if alibi else None)
    if prefix is not None:  # causal rows below R see only keys below R: an exact sub-problem
        R = prefix
        okw["bias"] = bias[..., :R, :R] if bias is not None else None
        o_ref, lse_ref = oracle.flash_fwd(q[:, :, :R], k[:, :, :R], v[:, :, :R], **okw)
        o, lse = o[:, :, :R], lse[:, :, :R]
    else:
        o_ref, lse_ref = oracle.flash_fwd(q, k, v, **okw)
    return {"case": name, "rc": rc, "check_bits": bits.value, "status": status, **parity(o, lse, o_ref, lse_ref)}


def main():
    rng = np.random.default_rng(5)
    cases = [
        ("single_tile_c1", dict(B=1, Hq=4, Hkv=4, M=512, N=512, D=64)),
        ("greedy_skipmax_causal_gqa", dict(B=1, Hq=16, Hkv=16, M=8192, N=8192, D=128, causal=True, prefix=384)),
        ("alibi_far_bound_m_ne_n", dict(B=2, Hq=4, Hkv=2, M=1000, N=900, D=128, causal=True,
                                         alibi_slopes=np.array([4.0, 1.0, 0.25, 0.0], np.float32))),
        ("alibi_softcap_c3_heads", dict(B=1, Hq=32, Hkv=32, M=2048, N=2048, D=128, causal=True, alibi=True,
                                        softcap=50.0, in_scale=0.5)),
        ("block_mask_bias", dict(B=2, Hq=4, Hkv=2, M=700, N=640, D=128, causal=True,
                                 block_mask=(rng.random((11, 10)) > 0.3).astype(np.uint8), mask_block=(64, 64),
                                 bias=rng.standard_normal((1, 1, 700, 640)).astype(np.float32))),
        ("d64_alibi_softcap", dict(B=2, Hq=8, Hkv=2, M=600, N=600, D=64, causal=True, alibi=True, softcap=20.0)),
        ("d64_dense_bias_full", dict(B=1, Hq=4, Hkv=4, M=300, N=500, D=64,
                                     bias=rng.standard_normal((1, 4, 300, 500)).astype(np.float32))),
        ("host_pieces_alibi", dict(B=1, Hq=16, Hkv=2, M=1024, N=1024, D=128, causal=True, alibi=True, entry="host")),
        ("host_chunks_dense", dict(B=2, Hq=8, Hkv=8, M=384, N=512, D=128, entry="host")),
        # KV splits: few items over long key ranges (split items, partial planes, merge)
        ("kv_splits_decode_gqa", dict(B=1, Hq=4, Hkv=1, M=100, N=3000, D=128)),
        ("kv_splits_causal_d64_softcap", dict(B=1, Hq=2, Hkv=2, M=256, N=2048, D=64, causal=True, softcap=20.0)),
        ("kv_splits_host", dict(B=1, Hq=4, Hkv=2, M=100, N=3000, D=128, entry="host")),
    ]
    for name, kw in cases:
        print(json.dumps(run_case(name, **kw)), flush=True)


if __name__ == "__main__":
    main()
