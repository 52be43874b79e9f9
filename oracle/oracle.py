"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` (as the checker) and bench.py's CPU
legs import this module.  It loads two libraries built by ``oracle/Makefile``:

* ``oracle/lib/libodf_oracle.so`` -- the C restatement of the reference's
  ``flash_attention_qk_pv_tile_ws`` (src/onednn_flash/attention.cpp:486-695)
  and ``standard_attention`` (attention.cpp:88-137), plus LSE, soft-cap, GQA
  and the tile (skip) map;
* ``oracle/_ref/libodf_ref.so`` -- the reference's own sources compiled
  unmodified, behind ``oracle/ref_shim.cpp``.  It exists only where the
  reference checkout was present at build time; ``ref_available()`` says so.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
ORACLE_LIB = _HERE / "lib" / "libodf_oracle.so"
REF_LIB = _HERE / "_ref" / "libodf_ref.so"
REF_BENCH = _HERE / "_ref" / "onednn_flash_bench"


class OracleParams(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
        ("o", C.c_void_p), ("lse", C.c_void_p),
        ("batch", C.c_int64), ("heads_q", C.c_int64), ("heads_kv", C.c_int64),
        ("m", C.c_int64), ("n", C.c_int64), ("d", C.c_int64), ("dv", C.c_int64),
        ("scale", C.c_float), ("causal", C.c_int),
        ("q_block", C.c_int64), ("k_block", C.c_int64),
        ("mask", C.c_void_p), ("mask_qbs", C.c_int64), ("mask_kbs", C.c_int64),
        ("mask_qblocks", C.c_int64), ("mask_kblocks", C.c_int64),
        ("alibi_slopes", C.c_void_p), ("softcap", C.c_float), ("nthreads", C.c_int),
        ("bias", C.c_void_p), ("bias_strides", C.c_int64 * 4),
    ]


_oracle = None
_ref = None


def _lib():
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            raise RuntimeError(f"oracle library missing: {ORACLE_LIB} (run __graft_entry__.build())")
        _oracle = C.CDLL(str(ORACLE_LIB))
        _oracle.odf_oracle_flash_fwd.argtypes = [C.POINTER(OracleParams)]
        _oracle.odf_oracle_standard_fwd.argtypes = [C.POINTER(OracleParams)]
        _oracle.odf_oracle_tile_map.argtypes = [C.c_int64] * 4 + [C.c_int, C.c_void_p] + [C.c_int64] * 4 + [C.c_void_p]
        _oracle.odf_oracle_round_bf16.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
    return _oracle


def ref_available() -> bool:
    return REF_LIB.exists()


def _reflib():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError(f"reference build missing: {REF_LIB}")
        _ref = C.CDLL(str(REF_LIB))
        for name in ("odf_ref_flash_ws", "odf_ref_standard", "odf_ref_tiled", "odf_ref_q_tile",
                     "odf_ref_qk_pv_tile", "odf_ref_batched"):
            getattr(_ref, name).argtypes = [C.POINTER(OracleParams)]
        _ref.odf_ref_score_mod_plan.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int,
                                                C.c_char_p, C.c_int]
        _ref.odf_ref_runtime_plan.argtypes = [C.POINTER(C.c_int), C.c_float, C.c_int, C.c_int,
                                              C.c_char_p, C.c_int]
        _ref.odf_ref_block_mask_plan.argtypes = [C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
        _ref.odf_ref_causal_mask_tile.argtypes = [C.c_int] * 4 + [C.c_char_p, C.c_int]
        _ref.odf_ref_backend_name.restype = C.c_char_p
        _ref.odf_ref_tile_kernel_name.restype = C.c_char_p
    return _ref


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 -> fp32 (values exactly representable in bf16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _lib().odf_oracle_round_bf16(x.ctypes.data, out.ctypes.data, x.size)
    return out


def _params(q, k, v, o, lse, *, scale, causal, q_block, k_block, mask, mask_block, alibi_slopes,
            softcap, nthreads, bias=None):
    B, Hq, M, D = q.shape
    _, Hkv, N, _ = k.shape
    DV = v.shape[3]
    p = OracleParams()
    p.q, p.k, p.v, p.o = q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data
    p.lse = lse.ctypes.data if lse is not None else None
    p.batch, p.heads_q, p.heads_kv, p.m, p.n, p.d, p.dv = B, Hq, Hkv, M, N, D, DV
    p.scale = scale
    p.causal = int(bool(causal))
    p.q_block, p.k_block = q_block, k_block
    if mask is not None:
        p.mask = mask.ctypes.data
        p.mask_qbs, p.mask_kbs = mask_block
        p.mask_qblocks, p.mask_kblocks = mask.shape
    p.alibi_slopes = alibi_slopes.ctypes.data if alibi_slopes is not None else None
    p.softcap = softcap
    p.nthreads = nthreads
    if bias is not None:  # float32 ndarray broadcastable to [B, Hq, M, N] (numpy strides, 0 = broadcast)
        bias = np.broadcast_to(bias, (B, Hq, M, N))
        p.bias = bias.ctypes.data
        for i in range(4):
            p.bias_strides[i] = bias.strides[i] // 4
    return p


def _prep(q, k, v, mask, alibi_slopes):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, v must be [B, H, T, D]")
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint8)
    if alibi_slopes is not None:
        alibi_slopes = np.ascontiguousarray(alibi_slopes, dtype=np.float32)
    return q, k, v, mask, alibi_slopes


def _run(fn_name, lib, q, k, v, *, scale=None, causal=False, q_block=128, k_block=128, mask=None,
         mask_block=(128, 128), alibi_slopes=None, softcap=0.0, want_lse=True, nthreads=None, bias=None):
    q, k, v, mask, alibi_slopes = _prep(q, k, v, mask, alibi_slopes)
    if bias is not None:
        bias = np.asarray(bias, dtype=np.float32)
    B, Hq, M, D = q.shape
    if scale is None:
        scale = 1.0 / float(np.sqrt(D))
    o = np.zeros((B, Hq, M, v.shape[3]), dtype=np.float32)
    lse = np.full((B, Hq, M), -np.inf, dtype=np.float32) if want_lse else None
    if nthreads is None:
        nthreads = max(1, min(os.cpu_count() or 1, 64))
    p = _params(q, k, v, o, lse, scale=scale, causal=causal, q_block=q_block, k_block=k_block, mask=mask,
                mask_block=mask_block, alibi_slopes=alibi_slopes, softcap=softcap, nthreads=nthreads, bias=bias)
    rc = getattr(lib, fn_name)(C.byref(p))
    if rc != 0:
        raise RuntimeError(f"{fn_name} failed with status {rc}")
    return o, lse


def flash_fwd(q, k, v, **kw):
    """Oracle flash forward (restatement).  Returns (O fp32 [B,Hq,M,Dv], LSE fp32 [B,Hq,M] or None)."""
    return _run("odf_oracle_flash_fwd", _lib(), q, k, v, **kw)


def standard_fwd(q, k, v, **kw):
    """Oracle materialising forward (restatement of standard_attention)."""
    return _run("odf_oracle_standard_fwd", _lib(), q, k, v, **kw)


def ref_fwd(variant, q, k, v, **kw):
    """Run the REFERENCE's own code: variant in {flash_ws, standard, tiled, q_tile, qk_pv_tile, batched}."""
    kw["want_lse"] = False
    o, _ = _run(f"odf_ref_{variant}", _reflib(), q, k, v, **kw)
    return o


def tile_map(m, n, bq, bk, causal, mask=None, mask_block=(128, 128)):
    """uint8 [ceil(m/bq), ceil(n/bk)]: 0 skipped, 1 full, 2 partial (element mask needed)."""
    nqt, nkt = -(-m // bq), -(-n // bk)
    out = np.zeros((nqt, nkt), dtype=np.uint8)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint8)
        rc = _lib().odf_oracle_tile_map(m, n, bq, bk, int(bool(causal)), mask.ctypes.data, mask_block[0],
                                        mask_block[1], mask.shape[0], mask.shape[1], out.ctypes.data)
    else:
        rc = _lib().odf_oracle_tile_map(m, n, bq, bk, int(bool(causal)), None, 0, 0, 0, 0, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"odf_oracle_tile_map failed with status {rc}")
    return out


def ref_score_mod_plan(kind, dtype, has_scale, scale, bias_kind, post_ops_available) -> str:
    buf = C.create_string_buffer(1024)
    _reflib().odf_ref_score_mod_plan(kind, dtype, int(has_scale), scale, bias_kind, int(post_ops_available), buf, 1024)
    return buf.value.decode()


def ref_runtime_plan(ints, scale, one_dnn_available, post_ops_available) -> str:
    arr = (C.c_int * 17)(*ints)
    buf = C.create_string_buffer(4096)
    _reflib().odf_ref_runtime_plan(arr, scale, int(one_dnn_available), int(post_ops_available), buf, 4096)
    return buf.value.decode()


def ref_block_mask_plan(kind, query_length, key_length) -> str:
    buf = C.create_string_buffer(1024)
    _reflib().odf_ref_block_mask_plan(kind, query_length, key_length, buf, 1024)
    return buf.value.decode()


def ref_causal_mask_tile(q_start, k_start, q_size, k_size) -> str:
    buf = C.create_string_buffer(1024)
    _reflib().odf_ref_causal_mask_tile(q_start, k_start, q_size, k_size, buf, 1024)
    return buf.value.decode()


def ref_backend_name(kind) -> str:
    return _reflib().odf_ref_backend_name(kind).decode()


def ref_tile_kernel_name(kind) -> str:
    return _reflib().odf_ref_tile_kernel_name(kind).decode()


def alibi_slopes(heads: int) -> np.ndarray:
    """Per-head ALiBi slopes 2^(-8 h / H) for h = 1..H (head index i uses h = i + 1)."""
    return np.array([2.0 ** (-8.0 * (i + 1) / heads) for i in range(heads)], dtype=np.float32)


def sliding_window_prefix_mask(n_blocks: int, window_blocks: int = 4, prefix_blocks: int = 4) -> np.ndarray:
    """Block mask allowed(qb, kb) = kb <= qb and (qb - kb < window_blocks or kb < prefix_blocks)."""
    qb = np.arange(n_blocks)[:, None]
    kb = np.arange(n_blocks)[None, :]
    return ((kb <= qb) & ((qb - kb < window_blocks) | (kb < prefix_blocks))).astype(np.uint8)
