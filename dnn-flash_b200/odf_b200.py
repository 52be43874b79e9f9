"""Python binding of the C ABI in include/odf_sm100.h (ctypes; torch tensors for device memory).

This module adds no compute of its own: every call goes through
``lib/libodf_sm100.so``.  If that library is missing the import fails loudly;
there is no CPU fallback.  Argument meaning and error behaviour follow the
reference's batched entry point ``flash_attention_batched_qk_pv_tile``
(src/onednn_flash/batched_attention.cpp:9-49): invalid sizes or null tensors
raise ``ValueError`` (the reference's ``std::invalid_argument``), anything the
GPU path cannot run raises ``RuntimeError`` (its ``std::runtime_error``).
"""
from __future__ import annotations

import ctypes as C
import math
import os
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "lib" / "libodf_sm100.so"
HEADER_PATHS = sorted((PACKAGE_DIR.parent / "include").glob("*.h"))

ODF_OK = 0
ODF_ERR_INVALID_ARG = 1
ODF_ERR_UNSUPPORTED = 2
ODF_ERR_CUDA = 3
ODF_ERR_DEVICE_TIMEOUT = 4
ODF_ERR_NO_DEVICE = 5
ODF_DTYPE_F32 = 0
ODF_DTYPE_BF16 = 1
ODF_BIAS_NONE = 0
ODF_BIAS_SAME_SHAPE = 1
ODF_BIAS_ALIBI = 4
TILE_Q = 128
TILE_K = 128


class FwdParams(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p), ("lse", C.c_void_p),
        ("qkv_dtype", C.c_int32), ("o_dtype", C.c_int32),
        ("batch", C.c_int64), ("heads_q", C.c_int64), ("heads_kv", C.c_int64),
        ("seqlen_q", C.c_int64), ("seqlen_k", C.c_int64), ("head_dim", C.c_int64), ("value_dim", C.c_int64),
        ("q_strides", C.c_int64 * 3), ("k_strides", C.c_int64 * 3), ("v_strides", C.c_int64 * 3),
        ("o_strides", C.c_int64 * 3),
        ("scale", C.c_float), ("causal", C.c_int32),
        ("block_mask", C.c_void_p), ("mask_qbs", C.c_int64), ("mask_kbs", C.c_int64),
        ("mask_qblocks", C.c_int64), ("mask_kblocks", C.c_int64),
        ("bias_kind", C.c_int32), ("alibi_slopes", C.c_void_p), ("softcap", C.c_float),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("tile_visits", C.c_void_p),
        ("bias", C.c_void_p), ("bias_strides", C.c_int64 * 4),
    ]


class OdfError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"odf status {code}: {message}")
        self.code = code


_lib = None


def load_library():
    """Load the sm_100a library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() (no CPU fallback exists)")
    lib = C.CDLL(str(LIB_PATH))
    lib.odf_flash_fwd_sm100.argtypes = [C.POINTER(FwdParams), C.c_void_p]
    lib.odf_flash_fwd_host.argtypes = [C.POINTER(FwdParams)]
    lib.odf_fwd_workspace_size.argtypes = [C.POINTER(FwdParams)]
    lib.odf_fwd_workspace_size.restype = C.c_size_t
    lib.odf_tile_map_sm100.argtypes = [C.c_int64, C.c_int64, C.c_int32, C.c_void_p, C.c_int64, C.c_int64,
                                       C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]
    lib.odf_convert_f32_to_bf16.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
    lib.odf_device_status.argtypes = [C.POINTER(C.c_int32), C.c_int32]
    lib.odf_last_error.restype = C.c_char_p
    lib.odf_version.restype = C.c_char_p
    _lib = lib
    return lib


def last_error() -> str:
    return load_library().odf_last_error().decode()


def version() -> str:
    return load_library().odf_version().decode()


def _check(rc: int):
    if rc == ODF_OK:
        return
    msg = last_error()
    if rc == ODF_ERR_INVALID_ARG:
        raise ValueError(f"odf status {rc}: {msg}")
    raise OdfError(rc, msg)


def declared_symbols() -> list[str]:
    """Every function name declared in include/*.h (the C ABI)."""
    import re

    names = []
    for path in HEADER_PATHS:
        text = path.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(odf_\w+)\s*\(", text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def alibi_slopes(heads: int) -> list[float]:
    """Generated ALiBi slopes 2^(-8 (h+1) / H), the values the kernel uses when none are given."""
    return [2.0 ** (-8.0 * (h + 1) / heads) for h in range(heads)]


def _strides4(t):
    s = t.stride()
    if s[3] != 1:
        raise ValueError("the innermost (feature) dimension must be contiguous")
    return (s[0], s[1], s[2])


def fill_params(q, k, v, o, lse, *, causal, scale, block_mask, mask_block, alibi, alibi_slopes_host, softcap,
                workspace, visits, bias=None) -> tuple[FwdParams, object]:
    """Populate odf_fwd_params from torch CUDA tensors; returns (params, keep-alive objects)."""
    import torch

    p = FwdParams()
    keep = []
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.qkv_dtype = ODF_DTYPE_BF16 if q.dtype == torch.bfloat16 else ODF_DTYPE_F32
    p.o_dtype = ODF_DTYPE_BF16 if o.dtype == torch.bfloat16 else ODF_DTYPE_F32
    B, Hq, M, D = q.shape
    _, Hkv, N, _ = k.shape
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k = B, Hq, Hkv, M, N
    p.head_dim, p.value_dim = D, v.shape[3]
    for name, t in (("q_strides", q), ("k_strides", k), ("v_strides", v), ("o_strides", o)):
        arr = getattr(p, name)
        for i, s in enumerate(_strides4(t)):
            arr[i] = s
    p.scale = scale
    p.causal = int(bool(causal))
    if block_mask is not None:
        p.block_mask = block_mask.data_ptr()
        p.mask_qbs, p.mask_kbs = mask_block
        p.mask_qblocks, p.mask_kblocks = block_mask.shape
    if alibi:
        p.bias_kind = ODF_BIAS_ALIBI
        if alibi_slopes_host is not None:
            arr = (C.c_float * len(alibi_slopes_host))(*[float(x) for x in alibi_slopes_host])
            keep.append(arr)
            p.alibi_slopes = C.cast(arr, C.c_void_p)
    p.softcap = softcap
    if bias is not None:
        if alibi:
            raise ValueError("ALiBi and a bias tensor are exclusive (one BiasKind per call)")
        # float32 CUDA tensor broadcastable to [B, Hq, M, N]; expand() gives 0 strides
        bias_v = bias.expand(B, Hq, M, N)
        p.bias_kind = ODF_BIAS_SAME_SHAPE
        p.bias = bias_v.data_ptr()
        for i, st in enumerate(bias_v.stride()):
            p.bias_strides[i] = st
        keep.append(bias_v)
    if workspace is not None:
        p.workspace = workspace.data_ptr()
        p.workspace_bytes = workspace.numel() * workspace.element_size()
    if visits is not None:
        p.tile_visits = visits.data_ptr()
    return p, keep


def flash_fwd(q, k, v, *, causal=False, scale=None, block_mask=None, mask_block=(128, 128), alibi=False,
              alibi_slopes=None, softcap=0.0, out_dtype=None, want_lse=True, out=None, lse_out=None,
              visits=None, stream=None, bias=None):
    """Forward pass on CUDA tensors q [B,Hq,M,D], k [B,Hkv,N,D], v [B,Hkv,N,Dv] (bf16).

    ``bias``: optional float32 CUDA tensor broadcastable to [B,Hq,M,N], added after the
    scale (BiasKind::SameShapeTile).

    Returns (o [B,Hq,M,Dv], lse [B,Hq,M] fp32 natural log, or None).  The launch
    is asynchronous on ``stream`` (default: torch's current stream).
    """
    import torch

    lib = load_library()
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be rank 4 [B, H, T, D]")
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[3])
    B, Hq, M, _ = q.shape
    dev = q.device
    if out is None:
        out = torch.empty((B, Hq, M, v.shape[3]), dtype=out_dtype or torch.float32, device=dev)
    lse = lse_out
    if want_lse and lse is None:
        lse = torch.empty((B, Hq, M), dtype=torch.float32, device=dev)
    mask_t = None
    if block_mask is not None:
        mask_t = torch.as_tensor(block_mask, dtype=torch.uint8).to(dev).contiguous()
    p, keep = fill_params(q, k, v, out, lse, causal=causal, scale=scale, block_mask=mask_t, mask_block=mask_block,
                          alibi=alibi, alibi_slopes_host=alibi_slopes, softcap=softcap, workspace=None,
                          visits=visits, bias=bias)
    ws_bytes = lib.odf_fwd_workspace_size(C.byref(p))
    ws = None
    if ws_bytes:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        p.workspace = ws.data_ptr()
        p.workspace_bytes = ws_bytes
    current = torch.cuda.current_stream(dev).cuda_stream
    if stream is None:
        stream = current
    _check(lib.odf_flash_fwd_sm100(C.byref(p), C.c_void_p(stream)))
    # Temporaries come from torch's allocator on the current stream; on another
    # stream they must outlive the launch, so wait for it before releasing them.
    if stream != current and (ws is not None or mask_t is not None):
        torch.cuda.synchronize(dev)
    del keep
    return out, (lse if want_lse else None)


def flash_fwd_host(q, k, v, *, causal=False, scale=None, block_mask=None, mask_block=(128, 128), alibi=False,
                   alibi_slopes=None, softcap=0.0, out=None, lse_out=None, bias=None):
    """Forward pass on HOST numpy buffers through odf_flash_fwd_host (blocking).

    q/k/v are float32 or bfloat16-as-uint16 arrays [B,H,T,D]; ``out`` (float32 or
    uint16 for bf16) and ``lse_out`` (float32 [B,Hq,M] or None) are filled in place.
    """
    import numpy as np

    lib = load_library()
    B, Hq, M, D = q.shape
    _, Hkv, N, _ = k.shape
    p = FwdParams()
    p.q, p.k, p.v = q.ctypes.data, k.ctypes.data, v.ctypes.data
    p.qkv_dtype = ODF_DTYPE_F32 if q.dtype == np.float32 else ODF_DTYPE_BF16
    if out is None:
        out = np.empty((B, Hq, M, v.shape[3]), dtype=np.float32)
    p.o = out.ctypes.data
    p.o_dtype = ODF_DTYPE_F32 if out.dtype == np.float32 else ODF_DTYPE_BF16
    p.lse = lse_out.ctypes.data if lse_out is not None else None
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim, p.value_dim = B, Hq, Hkv, M, N, D, v.shape[3]
    p.scale = (1.0 / math.sqrt(D)) if scale is None else scale
    p.causal = int(bool(causal))
    mask = None
    if block_mask is not None:
        mask = np.ascontiguousarray(block_mask, dtype=np.uint8)
        p.block_mask = mask.ctypes.data
        p.mask_qbs, p.mask_kbs = mask_block
        p.mask_qblocks, p.mask_kblocks = mask.shape
    keep = None
    if alibi:
        p.bias_kind = ODF_BIAS_ALIBI
        if alibi_slopes is not None:
            keep = (C.c_float * len(alibi_slopes))(*[float(x) for x in alibi_slopes])
            p.alibi_slopes = C.cast(keep, C.c_void_p)
    p.softcap = softcap
    bias_v = None
    if bias is not None:  # float32 array broadcastable to [B, Hq, M, N]
        bias_v = np.broadcast_to(np.asarray(bias, dtype=np.float32), (B, Hq, M, N))
        p.bias_kind = ODF_BIAS_SAME_SHAPE
        p.bias = bias_v.ctypes.data
        for i, st in enumerate(bias_v.strides):
            p.bias_strides[i] = st // 4
    _check(lib.odf_flash_fwd_host(C.byref(p)))
    del bias_v
    return out, lse_out


def tile_map(seqlen_q, seqlen_k, causal, block_mask=None, mask_block=(128, 128), device="cuda"):
    """Device tile map (uint8 [q_tiles, kv_tiles]: 0 skipped, 1 full, 2 element-masked)."""
    import torch

    lib = load_library()
    nqt, nkt = -(-seqlen_q // TILE_Q), -(-seqlen_k // TILE_K)
    out = torch.full((nqt, nkt), 255, dtype=torch.uint8, device=device)
    mask_t = None
    if block_mask is not None:
        mask_t = torch.as_tensor(block_mask, dtype=torch.uint8).to(device).contiguous()
        rc = lib.odf_tile_map_sm100(seqlen_q, seqlen_k, int(bool(causal)), mask_t.data_ptr(), mask_block[0],
                                    mask_block[1], mask_t.shape[0], mask_t.shape[1], out.data_ptr(),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream))
    else:
        rc = lib.odf_tile_map_sm100(seqlen_q, seqlen_k, int(bool(causal)), None, 0, 0, 0, 0, out.data_ptr(),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc)
    torch.cuda.synchronize()
    return out


def device_status(clear=True) -> int:
    v = C.c_int32(0)
    _check(load_library().odf_device_status(C.byref(v), int(clear)))
    return v.value


def env_threads() -> int:
    return max(1, min(os.cpu_count() or 1, 64))
