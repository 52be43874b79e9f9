"""CPU-only checks of the C ABI library: it loads, exports every symbol the
headers declare, and its host-side validation rejects bad arguments before any
CUDA call (no GPU needed for those paths)."""
from __future__ import annotations

import ctypes as C

import pytest

import odf_b200


def test_library_loads_and_reports_version():
    lib = odf_b200.load_library()
    assert "sm_100a" in odf_b200.version()
    assert lib is odf_b200.load_library()


def test_every_declared_symbol_is_exported():
    names = odf_b200.declared_symbols()
    expected = {"odf_flash_fwd_sm100", "odf_fwd_workspace_size", "odf_flash_fwd_host", "odf_tile_map_sm100",
                "odf_convert_f32_to_bf16", "odf_device_status", "odf_last_error", "odf_version"}
    assert expected <= set(names), f"headers lost a declaration: {expected - set(names)}"
    lib = odf_b200.load_library()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def _params(**over):
    p = odf_b200.FwdParams()
    dummy = 4096  # never dereferenced: validation fails first
    p.q = p.k = p.v = p.o = dummy
    p.qkv_dtype, p.o_dtype = odf_b200.ODF_DTYPE_BF16, odf_b200.ODF_DTYPE_F32
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim, p.value_dim = 1, 2, 2, 128, 128, 64, 64
    p.scale = 0.125
    for k, v in over.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("field,value,code", [
    ("q", None, odf_b200.ODF_ERR_INVALID_ARG),
    ("o", None, odf_b200.ODF_ERR_INVALID_ARG),
    ("batch", 0, odf_b200.ODF_ERR_INVALID_ARG),
    ("seqlen_k", 0, odf_b200.ODF_ERR_INVALID_ARG),
    ("heads_kv", 3, odf_b200.ODF_ERR_INVALID_ARG),
    ("head_dim", 96, odf_b200.ODF_ERR_UNSUPPORTED),
    ("value_dim", 128, odf_b200.ODF_ERR_UNSUPPORTED),
    ("qkv_dtype", odf_b200.ODF_DTYPE_F32, odf_b200.ODF_ERR_UNSUPPORTED),
    ("o_dtype", 7, odf_b200.ODF_ERR_UNSUPPORTED),
    ("softcap", -1.0, odf_b200.ODF_ERR_INVALID_ARG),
    ("scale", float("inf"), odf_b200.ODF_ERR_INVALID_ARG),
    ("bias_kind", odf_b200.ODF_BIAS_SAME_SHAPE, odf_b200.ODF_ERR_INVALID_ARG),  # SameShapeTile without a tensor
    ("bias_kind", 2, odf_b200.ODF_ERR_UNSUPPORTED),  # BiasKind::BroadcastRow: a strided SameShapeTile here
    ("seqlen_q", 65536 * 128, odf_b200.ODF_ERR_UNSUPPORTED),
])
def test_validation_codes(field, value, code):
    lib = odf_b200.load_library()
    rc = lib.odf_flash_fwd_sm100(C.byref(_params(**{field: value})), None)
    assert rc == code
    assert odf_b200.last_error()


def test_explicit_alibi_slopes_limited_to_256_heads():
    lib = odf_b200.load_library()
    slopes = (C.c_float * 300)()
    p = _params(bias_kind=odf_b200.ODF_BIAS_ALIBI, heads_q=300, heads_kv=300, alibi_slopes=C.cast(slopes, C.c_void_p))
    assert lib.odf_flash_fwd_sm100(C.byref(p), None) == odf_b200.ODF_ERR_UNSUPPORTED
    assert "256" in odf_b200.last_error()


def test_same_shape_bias_checks():
    lib = odf_b200.load_library()
    p = _params(bias_kind=odf_b200.ODF_BIAS_SAME_SHAPE, bias=4096)
    p.bias_strides[2] = -1
    assert lib.odf_flash_fwd_sm100(C.byref(p), None) == odf_b200.ODF_ERR_INVALID_ARG
    assert "stride" in odf_b200.last_error()
    p = _params(bias_kind=odf_b200.ODF_BIAS_SAME_SHAPE, bias=4098)
    assert lib.odf_flash_fwd_sm100(C.byref(p), None) == odf_b200.ODF_ERR_INVALID_ARG
    assert "aligned" in odf_b200.last_error()


def test_block_mask_needs_sizes_and_workspace():
    lib = odf_b200.load_library()
    p = _params(block_mask=4096)
    assert lib.odf_flash_fwd_sm100(C.byref(p), None) == odf_b200.ODF_ERR_INVALID_ARG
    p = _params(block_mask=4096, mask_qbs=128, mask_kbs=128, mask_qblocks=1, mask_kblocks=1)
    assert lib.odf_fwd_workspace_size(C.byref(p)) > 0
    assert lib.odf_flash_fwd_sm100(C.byref(p), None) == odf_b200.ODF_ERR_INVALID_ARG
    assert "workspace" in odf_b200.last_error()
    # without a mask the workspace only holds the work-item counter, and it stays optional
    assert lib.odf_fwd_workspace_size(C.byref(_params())) == 256
    small = _params(workspace=4096, workspace_bytes=64)
    assert lib.odf_flash_fwd_sm100(C.byref(small), None) == odf_b200.ODF_ERR_INVALID_ARG
    assert "smaller" in odf_b200.last_error()


def test_workspace_room_for_causal_alibi_far_bound():
    """Causal ALiBi at d = 128 asks for optional room after the 256-byte counter: per (batch,
    q-head) query-tile norms, per (batch, kv-head) KV-tile norms and per (batch, q-head) pair
    first KV tiles, int32/fp32 each, every array rounded up to 256 bytes.  Other shapes and
    masks do not; a 256-byte workspace stays valid (the bound is then left out)."""
    lib = odf_b200.load_library()
    up = lambda n: -(-n // 256) * 256
    B, Hq, Hkv, M, N = 2, 8, 2, 1000, 700
    nqt, nkt = -(-M // 128), -(-N // 128)
    npairs = -(-nqt // 2)
    base = dict(batch=B, heads_q=Hq, heads_kv=Hkv, seqlen_q=M, seqlen_k=N, head_dim=128, value_dim=128,
                causal=1, bias_kind=odf_b200.ODF_BIAS_ALIBI)
    want = 256 + up(B * Hq * nqt * 4) + up(B * Hkv * nkt * 4) + up(B * Hq * npairs * 4)
    assert lib.odf_fwd_workspace_size(C.byref(_params(**base))) == want
    assert lib.odf_fwd_workspace_size(C.byref(_params(**dict(base, causal=0)))) == 256
    assert lib.odf_fwd_workspace_size(C.byref(_params(**dict(base, head_dim=64, value_dim=64)))) == 256
    assert lib.odf_fwd_workspace_size(C.byref(_params(**dict(base, bias_kind=0)))) == 256


def _split_plan(B, Hq, M, N, sms=148):
    """The KV-split rule restated: (number of splits, KV tiles per split)."""
    nqt, nkt = -(-M // 128), -(-N // 128)
    single = nqt > 1 and B * Hq * nqt <= sms
    items = B * Hq * (nqt if single else -(-nqt // 2))
    s = min(sms // items, nkt // 4)  # at least four KV tiles per split
    if s < 2 or 2 * items > sms:
        return 1, nkt
    per = -(-nkt // s)
    return -(-nkt // per), per


def test_workspace_room_for_kv_splits():
    """Launches whose work items would leave more than half of a 148-SM GPU idle ask for optional
    room after the 256-byte counter for the fp32 partial O [splits, B, Hq, M, Dv] and LSE
    [splits, B, Hq, M] of their KV splits, each plane rounded up to 256 bytes.  Block masks, causal
    ALiBi at d = 128 and shapes with enough items ask for none."""
    lib = odf_b200.load_library()
    up = lambda n: -(-n // 256) * 256
    for B, Hq, Hkv, M, N, D, causal in [(1, 2, 1, 128, 4096, 128, 0), (1, 4, 4, 512, 2048, 64, 0),
                                         (2, 1, 1, 300, 1900, 128, 1), (1, 3, 3, 1, 4096, 64, 0)]:
        s, per = _split_plan(B, Hq, M, N)
        assert s > 1
        base = dict(batch=B, heads_q=Hq, heads_kv=Hkv, seqlen_q=M, seqlen_k=N, head_dim=D, value_dim=D,
                    causal=causal)
        want = 256 + up(s * B * Hq * M * D * 4) + up(s * B * Hq * M * 4)
        assert lib.odf_fwd_workspace_size(C.byref(_params(**base))) == want, (B, Hq, M, N, D)
    assert _split_plan(1, 4, 512, 512) == (1, 4)  # BASELINE c1: four KV tiles per query tile, too few to split
    assert _split_plan(1, 2, 128, 4096) == (8, 4)
    assert _split_plan(1, 8, 64, 32768) == (18, 15)
    assert _split_plan(8, 16, 4096, 4096) == (1, 32)  # c4: enough items, no splits
    # enough items, a block mask, or the causal ALiBi walk at d = 128: no split room
    big = dict(batch=8, heads_q=16, heads_kv=16, seqlen_q=2048, seqlen_k=2048, head_dim=128, value_dim=128)
    assert lib.odf_fwd_workspace_size(C.byref(_params(**big))) == 256
    dec = dict(batch=1, heads_q=2, heads_kv=2, seqlen_q=128, seqlen_k=4096, head_dim=128, value_dim=128)
    masked = _params(**dict(dec, block_mask=4096, mask_qbs=128, mask_kbs=128, mask_qblocks=1, mask_kblocks=32))
    nolist = lib.odf_fwd_workspace_size(C.byref(masked))
    assert nolist == 256 + up(1 * 32 * 4) + up(1 * 4)  # the tile lists alone
    walk = _params(**dict(dec, causal=1, bias_kind=odf_b200.ODF_BIAS_ALIBI))
    nqt, nkt = 1, 32
    assert lib.odf_fwd_workspace_size(C.byref(walk)) == 256 + up(2 * nqt * 4) + up(2 * nkt * 4) + up(2 * 1 * 4)


def test_misaligned_device_pointer_rejected():
    lib = odf_b200.load_library()
    assert lib.odf_flash_fwd_sm100(C.byref(_params(q=4096 + 2)), None) == odf_b200.ODF_ERR_INVALID_ARG


def test_null_params_and_status_pointer():
    lib = odf_b200.load_library()
    assert lib.odf_flash_fwd_sm100(None, None) == odf_b200.ODF_ERR_INVALID_ARG
    assert lib.odf_device_status(None, 0) == odf_b200.ODF_ERR_INVALID_ARG
    assert lib.odf_tile_map_sm100(10, 10, 1, None, 0, 0, 0, 0, None, None) == odf_b200.ODF_ERR_INVALID_ARG


def test_declared_symbols_parser_sees_all_headers():
    assert odf_b200.HEADER_PATHS, "include/*.h missing"
    assert all(n.startswith("odf_") for n in odf_b200.declared_symbols())


def test_debug_wait_hook_validation():
    """odf_debug_set_wait takes 0 (default) or a limit within [1 ms, 60 s], and -1 (off) or a
    load index; it only sets this thread's launch options (no CUDA call)."""
    lib = odf_b200.load_library()
    lib.odf_debug_set_wait.argtypes = [C.c_uint64, C.c_int32]
    assert lib.odf_debug_set_wait(500_000, -1) == odf_b200.ODF_ERR_INVALID_ARG
    assert "limit" in odf_b200.last_error()
    assert lib.odf_debug_set_wait(61_000_000_000, -1) == odf_b200.ODF_ERR_INVALID_ARG
    assert lib.odf_debug_set_wait(20_000_000, -2) == odf_b200.ODF_ERR_INVALID_ARG
    assert lib.odf_debug_set_wait(20_000_000, 3) == odf_b200.ODF_OK
    assert lib.odf_debug_set_wait(0, -1) == odf_b200.ODF_OK
