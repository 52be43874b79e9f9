"""Pins the CPU oracle to the reference itself (oracle/_ref is the reference's own
sources compiled unmodified).  With the features the reference has (scale, causal,
BlockMask, additive ALiBi bias through ScoreBiasFn, any tile sizes, GQA via per-head
pointers) the restatement must equal the reference bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import make_qkv

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference build (oracle/_ref) not present")


@needs_ref
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("tiles", [(1, 64), (16, 32), (128, 128), (7, 13), (64, 1)])
def test_ws_path_bit_exact(causal, tiles):
    q, k, v = make_qkv(21, 1, 2, 2, 150, 170, 32)
    o, _ = oracle.flash_fwd(q, k, v, causal=causal, q_block=tiles[0], k_block=tiles[1])
    r = oracle.ref_fwd("flash_ws", q, k, v, causal=causal, q_block=tiles[0], k_block=tiles[1])
    assert np.array_equal(o, r)


@needs_ref
def test_alibi_blockmask_gqa_bit_exact():
    rng = np.random.default_rng(5)
    q, k, v = make_qkv(22, 2, 4, 2, 200, 190, 64)
    mask = (rng.random((4, 7)) > 0.3).astype(np.uint8)
    slopes = oracle.alibi_slopes(4)
    kw = dict(causal=True, q_block=32, k_block=64, mask=mask, mask_block=(64, 32), alibi_slopes=slopes)
    o, _ = oracle.flash_fwd(q, k, v, **kw)
    r = oracle.ref_fwd("flash_ws", q, k, v, **kw)
    assert np.array_equal(o, r)


@needs_ref
@pytest.mark.parametrize("layout", ["full", "head_broadcast", "key_row", "strided"])
@pytest.mark.parametrize("causal", [False, True])
def test_bias_tensor_bit_exact(layout, causal):
    """The oracle's strided bias tensor (BiasKind::SameShapeTile on the GPU) equals the reference
    given the same values through its ScoreBiasFn (attention.cpp:619), for the flash and the
    materialising paths."""
    rng = np.random.default_rng(7)
    B, H, M, N = 2, 3, 150, 170
    q, k, v = make_qkv(26, B, H, H, M, N, 32)
    if layout == "full":
        bias = rng.standard_normal((B, H, M, N)).astype(np.float32)
    elif layout == "head_broadcast":
        bias = rng.standard_normal((1, 1, M, N)).astype(np.float32)
    elif layout == "key_row":
        bias = rng.standard_normal((1, 1, 1, N)).astype(np.float32)
    else:
        bias = rng.standard_normal((B, H, M, 2 * N)).astype(np.float32)[..., ::2]
    kw = dict(causal=causal, q_block=16, k_block=32, bias=bias)
    o, _ = oracle.flash_fwd(q, k, v, **kw)
    assert np.array_equal(o, oracle.ref_fwd("flash_ws", q, k, v, **kw))
    s, _ = oracle.standard_fwd(q, k, v, causal=causal, bias=bias)
    assert np.array_equal(s, oracle.ref_fwd("standard", q, k, v, causal=causal, bias=bias))


@needs_ref
@pytest.mark.parametrize("variant", ["standard", "tiled", "q_tile", "qk_pv_tile"])
def test_other_reference_entry_points_agree(variant):
    """standard_attention / flash_attention_tiled / _q_tile / _qk_pv_tile (attention.cpp:88-484)."""
    q, k, v = make_qkv(23, 1, 2, 2, 130, 140, 64)
    o, _ = oracle.flash_fwd(q, k, v, causal=True, q_block=16, k_block=32)
    r = oracle.ref_fwd(variant, q, k, v, causal=True, q_block=16, k_block=32)
    assert np.abs(o - r).max() <= 1e-6
    if variant == "standard":
        s, _ = oracle.standard_fwd(q, k, v, causal=True)
        assert np.array_equal(s, r)


@needs_ref
def test_batched_driver_as_shipped():
    """flash_attention_batched_qk_pv_tile (batched_attention.cpp:9-49), serial, as shipped."""
    q, k, v = make_qkv(24, 2, 3, 3, 96, 96, 64)
    o, _ = oracle.flash_fwd(q, k, v, causal=True, q_block=16, k_block=32)
    r = oracle.ref_fwd("batched", q, k, v, causal=True, q_block=16, k_block=32)
    assert np.array_equal(o, r)


@needs_ref
def test_fully_masked_rows_stay_unwritten_in_reference():
    """Rows with l <= 0 are left as the caller initialised them (attention.cpp:680-682)."""
    q, k, v = make_qkv(25, 1, 1, 1, 64, 64, 32)
    mask = np.array([[1, 1], [0, 0]], dtype=np.uint8)
    r = oracle.ref_fwd("flash_ws", q, k, v, mask=mask, mask_block=(32, 32))
    o, lse = oracle.flash_fwd(q, k, v, mask=mask, mask_block=(32, 32))
    assert np.all(r[0, 0, 32:] == 0) and np.all(o[0, 0, 32:] == 0)
    assert np.all(np.isneginf(lse[0, 0, 32:]))
    assert np.array_equal(o, r)


def test_lse_definition():
    """LSE = m + ln(l) equals log(sum(exp(s))) of the materialised scores."""
    q, k, v = make_qkv(26, 1, 1, 1, 40, 50, 16)
    _, lse = oracle.flash_fwd(q, k, v, causal=True, q_block=8, k_block=16)
    s = (q[0, 0].astype(np.float64) @ k[0, 0].astype(np.float64).T) / 4.0
    s = np.where(np.arange(50)[None, :] > np.arange(40)[:, None], -np.inf, s)
    ref = np.log(np.exp(s - s.max(1, keepdims=True)).sum(1)) + s.max(1)
    assert np.abs(lse[0, 0] - ref).max() < 1e-5


def test_softcap_matches_float64():
    q, k, v = make_qkv(27, 1, 1, 1, 33, 47, 16, scale=3.0)
    o, lse = oracle.flash_fwd(q, k, v, softcap=5.0, q_block=16, k_block=16)
    s = (q[0, 0].astype(np.float64) @ k[0, 0].astype(np.float64).T) / 4.0
    s = 5.0 * np.tanh(s / 5.0)
    p = np.exp(s - s.max(1, keepdims=True))
    ref = (p @ v[0, 0].astype(np.float64)) / p.sum(1, keepdims=True)
    assert np.abs(o[0, 0] - ref).max() < 1e-5


def test_tile_map_matches_reference_causal_break():
    """Skip rule = the reference's causal break k_begin >= q_end (attention.cpp:537-539)."""
    for m, n, bq, bk in [(1000, 1000, 128, 128), (700, 1300, 128, 128), (130, 70, 16, 32), (1, 5, 128, 128)]:
        tm = oracle.tile_map(m, n, bq, bk, True)
        for qt in range(tm.shape[0]):
            q_end = min(m, (qt + 1) * bq)
            for kt in range(tm.shape[1]):
                assert (tm[qt, kt] == 0) == (kt * bk >= q_end)


def test_c4_mask_density():
    mask = oracle.sliding_window_prefix_mask(32)
    assert int(mask.sum()) == 228
    tm = oracle.tile_map(4096, 4096, 128, 128, True, mask, (128, 128))
    assert int((tm != 0).sum()) == 228
    assert int((tm == 2).sum()) == 32  # the diagonal tiles need the element-level causal mask
