"""GPU parity: the sm_100a kernel (through the C ABI) against the CPU oracle.

Tolerances (bf16 Q/K/V, fp32 accumulation, compared in fp32):
  O   relative-L2 <= 1e-2 and max-abs <= 2e-2
  LSE max-abs    <= 1e-3
  skipped tile set: bit-exact.
The oracle restates the reference's flash_attention_qk_pv_tile_ws
(src/onednn_flash/attention.cpp:486-695); its agreement with the reference
itself is pinned by tests/test_oracle_vs_reference.py.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import make_qkv

pytestmark = pytest.mark.gpu

O_REL_L2 = 1e-2
O_MAX_ABS = 2e-2
LSE_MAX_ABS = 1e-3


def _torch():
    import torch

    return torch


def to_dev(x, dtype=None):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda").to(dtype or torch.bfloat16)


def run_gpu(q, k, v, **kw):
    import odf_b200

    torch = _torch()
    o, lse = odf_b200.flash_fwd(to_dev(q), to_dev(k), to_dev(v), **kw)
    torch.cuda.synchronize()
    return o.float().cpu().numpy(), (lse.cpu().numpy() if lse is not None else None)


def check_close(o, lse, o_ref, lse_ref, what=""):
    assert np.all(np.isfinite(o)), f"{what}: non-finite output"
    diff = o.astype(np.float64) - o_ref.astype(np.float64)
    denom = max(np.linalg.norm(o_ref.astype(np.float64)), 1e-30)
    rel = np.linalg.norm(diff) / denom
    mx = np.abs(diff).max()
    assert rel <= O_REL_L2, f"{what}: O rel-L2 {rel:.3e}"
    assert mx <= O_MAX_ABS, f"{what}: O max-abs {mx:.3e}"
    if lse is not None and lse_ref is not None:
        fin = np.isfinite(lse_ref)
        assert np.array_equal(np.isfinite(lse), fin), f"{what}: LSE -inf pattern differs"
        if fin.any():
            e = np.abs(lse[fin] - lse_ref[fin]).max()
            assert e <= LSE_MAX_ABS, f"{what}: LSE max-abs {e:.3e}"


def oracle_fwd(q, k, v, **kw):
    import oracle

    return oracle.flash_fwd(q, k, v, **kw)


# --------------------------------------------------------------------------- BASELINE configs
def test_config1_noncausal_d64():
    """c1: B1 H4 N512 d64, no mask, fp32 O."""
    q, k, v = make_qkv(1, 1, 4, 4, 512, 512, 64)
    o, lse = run_gpu(q, k, v)
    o_ref, lse_ref = oracle_fwd(q, k, v, q_block=16, k_block=32)
    check_close(o, lse, o_ref, lse_ref, "c1")


def test_config2_causal_d64():
    """c2: B4 H16 N2048 d64 causal, fp32 O + LSE (full size)."""
    q, k, v = make_qkv(2, 4, 16, 16, 2048, 2048, 64)
    o, lse = run_gpu(q, k, v, causal=True)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True)
    check_close(o, lse, o_ref, lse_ref, "c2")


def test_config3_alibi_softcap_reduced():
    """c3 at reduced length with the config's 32 heads (so the slopes are c3's 2^(-8h/32)):
    causal + ALiBi + soft-cap 50, inputs N(0,1)*0.5, bf16 O."""
    torch = _torch()
    import oracle

    H = 32
    q, k, v = make_qkv(3, 1, H, H, 1024, 1024, 128, scale=0.5)
    o, lse = run_gpu(q, k, v, causal=True, alibi=True, softcap=50.0, out_dtype=torch.bfloat16)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, alibi_slopes=oracle.alibi_slopes(H), softcap=50.0)
    check_close(o, lse, o_ref, lse_ref, "c3-reduced")


def test_config4_block_sparse_reduced():
    """c4 at reduced length: 128x128 sliding-window(4 blocks)+prefix(4 blocks) mask with causal."""
    import oracle

    nb = 12
    mask = oracle.sliding_window_prefix_mask(nb)
    q, k, v = make_qkv(4, 2, 2, 2, nb * 128, nb * 128, 128)
    o, lse = run_gpu(q, k, v, causal=True, block_mask=mask, mask_block=(128, 128))
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, mask=mask, mask_block=(128, 128))
    check_close(o, lse, o_ref, lse_ref, "c4-reduced")


def test_config5_gqa_reduced():
    """c5 at reduced length: GQA Hq=16, Hkv=2, causal, bf16 O + fp32 LSE."""
    torch = _torch()
    q, k, v = make_qkv(5, 1, 16, 2, 1024, 1024, 128)
    o, lse = run_gpu(q, k, v, causal=True, out_dtype=torch.bfloat16)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True)
    check_close(o, lse, o_ref, lse_ref, "c5-reduced")


# --------------------------------------------------------------------------- edge cases
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("n", [1, 127, 128, 129, 257])
def test_ragged_lengths(n, causal, d):
    q, k, v = make_qkv(100 + n, 1, 2, 2, n, n, d)
    o, lse = run_gpu(q, k, v, causal=causal)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=causal)
    check_close(o, lse, o_ref, lse_ref, f"n={n} causal={causal} d={d}")


@pytest.mark.parametrize("m,n", [(200, 70), (70, 300), (1, 513), (300, 1)])
@pytest.mark.parametrize("causal", [False, True])
def test_m_ne_n_top_left_causal(m, n, causal):
    """M != N: causal stays top-left aligned (kj > qi masked), as attention.cpp:55."""
    q, k, v = make_qkv(7, 1, 3, 3, m, n, 64)
    o, lse = run_gpu(q, k, v, causal=causal)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=causal)
    check_close(o, lse, o_ref, lse_ref, f"m={m} n={n}")


def test_fully_masked_rows_zero_and_neg_inf_lse():
    """A query block with no allowed key block: O rows are 0, LSE is -inf."""
    mask = np.ones((3, 3), dtype=np.uint8)
    mask[1, :] = 0
    q, k, v = make_qkv(8, 1, 2, 2, 300, 300, 64)
    o, lse = run_gpu(q, k, v, block_mask=mask, mask_block=(128, 128))
    o_ref, lse_ref = oracle_fwd(q, k, v, mask=mask, mask_block=(128, 128))
    assert np.all(o[:, :, 128:256] == 0.0)
    assert np.all(np.isneginf(lse[:, :, 128:256]))
    check_close(o, lse, o_ref, lse_ref, "masked rows")


@pytest.mark.parametrize("mask_block", [(64, 64), (128, 256), (32, 96), (200, 50)])
def test_block_mask_sizes_independent_of_tiles(mask_block):
    """BlockMask block sizes need not match the 128x128 tiles (attention.cpp:70-86)."""
    rng = np.random.default_rng(9)
    M = N = 520
    mqb, mkb = -(-M // mask_block[0]), -(-N // mask_block[1])
    mask = (rng.random((mqb, mkb)) > 0.35).astype(np.uint8)
    q, k, v = make_qkv(10, 1, 2, 2, M, N, 64)
    o, lse = run_gpu(q, k, v, causal=True, block_mask=mask, mask_block=mask_block)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, mask=mask, mask_block=mask_block)
    check_close(o, lse, o_ref, lse_ref, f"mask {mask_block}")


def test_block_mask_smaller_than_sequence_disallows_rest():
    """Blocks outside the bitmap are disallowed (attention.cpp:82-84)."""
    mask = np.ones((2, 2), dtype=np.uint8)
    q, k, v = make_qkv(11, 1, 1, 1, 400, 400, 64)
    o, lse = run_gpu(q, k, v, block_mask=mask, mask_block=(128, 128))
    o_ref, lse_ref = oracle_fwd(q, k, v, mask=mask, mask_block=(128, 128))
    check_close(o, lse, o_ref, lse_ref, "short bitmap")


@pytest.mark.parametrize("softcap", [0.0, 5.0, 50.0])
@pytest.mark.parametrize("alibi", [False, True])
def test_score_mods(alibi, softcap):
    import oracle

    H = 4
    q, k, v = make_qkv(12, 2, H, H, 384, 384, 128, scale=1.5)
    o, lse = run_gpu(q, k, v, causal=True, alibi=alibi, softcap=softcap)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, alibi_slopes=oracle.alibi_slopes(H) if alibi else None,
                                softcap=softcap)
    check_close(o, lse, o_ref, lse_ref, f"alibi={alibi} softcap={softcap}")


@pytest.mark.parametrize("softcap", [0.0, 30.0])
def test_generated_alibi_slopes_beyond_256_heads(softcap):
    """Up to 256 heads the host evaluates the generated slopes 2^(-8(h+1)/H) into the launch;
    beyond that the kernel evaluates them itself.  320 q-heads over 40 kv-heads (GQA 8)."""
    import oracle

    H, Hk = 320, 40
    q, k, v = make_qkv(41, 1, H, Hk, 200, 200, 64)
    o, lse = run_gpu(q, k, v, causal=True, alibi=True, softcap=softcap)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, alibi_slopes=oracle.alibi_slopes(H), softcap=softcap)
    check_close(o, lse, o_ref, lse_ref, f"generated slopes, 320 heads, softcap {softcap}")


@pytest.mark.parametrize("m,n", [(1000, 1000), (300, 700), (700, 300), (129, 129)])
@pytest.mark.parametrize("softcap", [0.0, 20.0])
def test_causal_alibi_far_tiles_diagonal_first(m, n, softcap):
    """Causal ALiBi at d = 128 walks each query tile's KV tiles from the diagonal down to tile 0,
    and a tile whose scores all lie 48 (log2) below the running max writes P = 0 without the
    exponentials.  Steep slopes make most tiles far; GQA, ragged ends and M != N (top-left causal)
    cross the pair and row bookkeeping of the reversed walk."""
    H, Hk = 4, 2
    slopes = np.array([4.0, 1.0, 0.25, 0.0625], dtype=np.float32)
    q, k, v = make_qkv(61, 2, H, Hk, m, n, 128)
    o, lse = run_gpu(q, k, v, causal=True, alibi=True, alibi_slopes=slopes, softcap=softcap)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, alibi_slopes=slopes, softcap=softcap)
    check_close(o, lse, o_ref, lse_ref, f"far tiles m={m} n={n} softcap={softcap}")


@pytest.mark.parametrize("softcap,in_scale", [(0.0, 1.0), (50.0, 0.5)])
def test_causal_alibi_norm_bound_leaves_out_only_far_tiles(softcap, in_scale):
    """Causal ALiBi at d = 128 with a workspace: KV tiles that a Cauchy-Schwarz bound on the
    tile norms shows to be far (every score below the row max by more than 48 ln 2) are not
    visited at all.  Every tile left out must be far in float64 on the actual scores; a zero
    slope leaves out nothing; steep slopes leave out most tiles; O and LSE match the oracle."""
    torch = _torch()
    import odf_b200
    import oracle

    H, M = 3, 1024
    slopes = np.array([2.0, 0.25, 0.0], dtype=np.float32)
    q, k, v = make_qkv(71, 1, H, H, M, M, 128, scale=in_scale)
    nt = M // 128
    visits = torch.zeros((H, nt, nt), dtype=torch.uint8, device="cuda")
    o, lse = odf_b200.flash_fwd(to_dev(q), to_dev(k), to_dev(v), causal=True, alibi=True, alibi_slopes=slopes,
                                softcap=softcap, visits=visits)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, alibi_slopes=slopes, softcap=softcap)
    check_close(o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, f"norm bound softcap={softcap}")

    causal_map = oracle.tile_map(M, M, 128, 128, True, None, (128, 128)) != 0
    processed = visits.cpu().numpy() != 0
    assert np.array_equal(processed[2], causal_map), "zero slope: a tile was left out"
    # slope 2: a KV tile two or more below a pair's first query tile is 258+ keys away (a bound
    # of -500 against a margin of about 70), so each pair keeps only its band of three tiles
    for qt in range(2, nt):
        assert not processed[0, qt, :2 * (qt // 2) - 1].any(), f"steep slope: query tile {qt} visited a far tile"
    scale = 1.0 / math.sqrt(128)
    ii, jj = np.meshgrid(np.arange(M), np.arange(M), indexing="ij")
    for h in range(H):
        t = (q[0, h].astype(np.float64) @ k[0, h].astype(np.float64).T) * scale + float(slopes[h]) * (jj - ii)
        if softcap > 0.0:
            t = softcap * np.tanh(t / softcap)
        t = np.where(jj <= ii, t, -np.inf)
        row_max = t.max(axis=1, keepdims=True)
        for qt in range(nt):
            for kt in range(nt):
                if causal_map[qt, kt] and not processed[h, qt, kt]:
                    gap = (t[qt * 128:(qt + 1) * 128, kt * 128:(kt + 1) * 128] - row_max[qt * 128:(qt + 1) * 128]).max()
                    assert gap < -48.0 * math.log(2.0), f"head {h} tile ({qt},{kt}) left out at gap {gap:.2f}"


def test_explicit_alibi_slopes_and_noncausal_scale():
    H = 3
    slopes = np.array([0.5, 0.03125, 0.25], dtype=np.float32)
    q, k, v = make_qkv(13, 1, H, H, 260, 300, 64)
    o, lse = run_gpu(q, k, v, scale=0.3, alibi=True, alibi_slopes=slopes)
    o_ref, lse_ref = oracle_fwd(q, k, v, scale=0.3, alibi_slopes=slopes)
    check_close(o, lse, o_ref, lse_ref, "explicit slopes")


def test_strided_bmhd_layout_and_bf16_output():
    """Q/K/V/O given as [B, T, H, D] memory (permuted views), bf16 output."""
    torch = _torch()
    import odf_b200

    B, H, M, D = 2, 4, 300, 128
    q, k, v = make_qkv(14, B, H, H, M, M, D)
    qd = to_dev(q.transpose(0, 2, 1, 3)).permute(0, 2, 1, 3)
    kd = to_dev(k.transpose(0, 2, 1, 3)).permute(0, 2, 1, 3)
    vd = to_dev(v.transpose(0, 2, 1, 3)).permute(0, 2, 1, 3)
    out = torch.empty((B, M, H, D), dtype=torch.bfloat16, device="cuda").permute(0, 2, 1, 3)
    o, lse = odf_b200.flash_fwd(qd, kd, vd, causal=True, out=out)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True)
    check_close(o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, "strided")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("o_dtype", ["float32", "bfloat16"])
def test_output_writes_stay_inside_o(d, o_dtype):
    """O is a view into a larger buffer (rows past M, columns past D): the padding keeps its
    sentinel, so the epilogue writes exactly rows < M and columns < D of every (batch, head)."""
    torch = _torch()
    import odf_b200

    B, H, M = 2, 3, 300
    dt = getattr(torch, o_dtype)
    q, k, v = make_qkv(31 + d, B, H, H, M, M, d)
    big = torch.full((B, H, M + 70, d + 24), -7.0, dtype=dt, device="cuda")
    out = big[:, :, :M, :d]
    o, lse = odf_b200.flash_fwd(to_dev(q), to_dev(k), to_dev(v), causal=True, out=out)
    torch.cuda.synchronize()
    assert o.data_ptr() == out.data_ptr()
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True)
    check_close(out.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, f"padded O {o_dtype} d={d}")
    pad = big.float().cpu().numpy()
    assert np.all(pad[:, :, M:, :] == -7.0), "rows past M were written"
    assert np.all(pad[:, :, :, d:] == -7.0), "columns past D were written"


# --------------------------------------------------------------------------- skip set
@pytest.mark.parametrize("case", ["causal", "mask", "mask_causal", "ragged"])
def test_skip_set_bit_exact(case):
    """The tiles the kernel processes equal the oracle's non-skipped tiles, bit for bit."""
    torch = _torch()
    import odf_b200
    import oracle

    M, N, causal, mask, mb = 1000, 1000, False, None, (128, 128)
    if case == "causal":
        causal = True
    elif case == "mask":
        mask = oracle.sliding_window_prefix_mask(8)
    elif case == "mask_causal":
        causal, mask, mb = True, oracle.sliding_window_prefix_mask(16, 3, 2), (64, 64)
    else:
        M, N, causal = 700, 1300, True
    q, k, v = make_qkv(15, 1, 2, 2, M, N, 64)
    nqt, nkt = -(-M // 128), -(-N // 128)
    visits = torch.zeros((2, nqt, nkt), dtype=torch.uint8, device="cuda")
    odf_b200.flash_fwd(to_dev(q), to_dev(k), to_dev(v), causal=causal, block_mask=mask, mask_block=mb,
                       visits=visits)
    torch.cuda.synchronize()
    ref_map = oracle.tile_map(M, N, 128, 128, causal, mask, mb)
    dev_map = odf_b200.tile_map(M, N, causal, mask, mb).cpu().numpy()
    assert np.array_equal(dev_map, ref_map), "device tile map differs from the oracle"
    processed = visits.cpu().numpy()
    for h in range(2):
        assert np.array_equal(processed[h] != 0, ref_map != 0), f"head {h}: processed set differs"


def test_config4_full_size_skip_density():
    """c4 geometry: 32x32 blocks, 228 allowed (22.3%); the kernel visits exactly those tiles."""
    torch = _torch()
    import odf_b200
    import oracle

    mask = oracle.sliding_window_prefix_mask(32)
    assert int(mask.sum()) == 228
    ref_map = oracle.tile_map(4096, 4096, 128, 128, True, mask, (128, 128))
    assert int((ref_map != 0).sum()) == 228
    dev_map = odf_b200.tile_map(4096, 4096, True, mask, (128, 128)).cpu().numpy()
    assert np.array_equal(dev_map, ref_map)


# --------------------------------------------------------------------------- full-size properties
def _dense_rows_f64(q, k, v, rows, *, causal, scale, slopes=None, softcap=0.0):
    """float64 reference for a few query rows of one head (independent numpy restatement)."""
    qr = q[rows].astype(np.float64)
    s = qr @ k.astype(np.float64).T * scale
    kj = np.arange(k.shape[0])[None, :]
    qi = np.asarray(rows)[:, None]
    if slopes is not None:
        s = s + slopes * (kj - qi)
    if softcap > 0:
        s = softcap * np.tanh(s / softcap)
    if causal:
        s = np.where(kj > qi, -np.inf, s)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    return (p @ v.astype(np.float64)) / l, (m + np.log(l))[:, 0]


def test_config3_full_size_rows():
    """c3 at full size (B2 H32 N8192 d128, ALiBi + soft-cap 50): sampled rows vs a float64 restatement."""
    torch = _torch()
    import odf_b200

    B, H, N, D = 2, 32, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(33)
    q = (torch.randn((B, H, N, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, H, N, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, H, N, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    o, lse = odf_b200.flash_fwd(q, k, v, causal=True, alibi=True, softcap=50.0, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    slopes = odf_b200.alibi_slopes(H)
    rows = [0, 1, 127, 128, 4095, 8191]
    for b, h in [(0, 0), (1, 31), (0, 17)]:
        qh, kh, vh = (t[b, h].float().cpu().numpy() for t in (q, k, v))
        o_ref, lse_ref = _dense_rows_f64(qh, kh, vh, rows, causal=True, scale=1 / math.sqrt(D), slopes=slopes[h],
                                         softcap=50.0)
        got = o[b, h, rows].float().cpu().numpy()
        assert np.abs(got - o_ref).max() <= O_MAX_ABS
        assert np.abs(lse[b, h, rows].cpu().numpy() - lse_ref).max() <= LSE_MAX_ABS


def test_config3_full_size_prefix_vs_oracle():
    """c3 at full size (B2 H32 N8192 d128, ALiBi 2^(-8h/32) + soft-cap 50, inputs N(0,1)*0.5,
    bf16 O): causal rows < R see only keys < R, so the prefix [0, R) of four (batch, head) units
    is an exact sub-problem, checked against the oracle with those heads' slopes."""
    torch = _torch()
    import odf_b200
    import oracle

    B, H, N, D = 2, 32, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(34)
    q, k, v = ((torch.randn((B, H, N, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16) for _ in range(3))
    o, lse = odf_b200.flash_fwd(q, k, v, causal=True, alibi=True, softcap=50.0, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    R = 768
    units = [(0, 0), (1, 31), (0, 17), (1, 6)]
    slopes = oracle.alibi_slopes(H)
    sel = lambda t: np.stack([t[b, h, :R].float().cpu().numpy() for b, h in units])[None]
    o_ref, lse_ref = oracle_fwd(sel(q), sel(k), sel(v), causal=True,
                                alibi_slopes=np.float32([slopes[h] for _, h in units]), softcap=50.0)
    check_close(sel(o), np.stack([lse[b, h, :R].cpu().numpy() for b, h in units])[None], o_ref, lse_ref,
                "c3 full-size prefix")


def test_config4_full_size_units_vs_oracle():
    """c4 at full size (B8 H16 N4096 d128, 128x128 window-4 + prefix-4 block mask with causal,
    22.3% of the blocks): every row of three (batch, head) units against the oracle."""
    torch = _torch()
    import odf_b200
    import oracle

    B, H, N, D = 8, 16, 4096, 128
    mask = oracle.sliding_window_prefix_mask(N // 128)
    g = torch.Generator(device="cuda").manual_seed(44)
    q, k, v = (torch.randn((B, H, N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    o, lse = odf_b200.flash_fwd(q, k, v, causal=True, block_mask=mask, mask_block=(128, 128),
                                out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    units = [(0, 0), (3, 7), (7, 15)]
    sel = lambda t: np.stack([t[b, h].float().cpu().numpy() for b, h in units])[None]
    o_ref, lse_ref = oracle_fwd(sel(q), sel(k), sel(v), causal=True, mask=mask, mask_block=(128, 128))
    check_close(sel(o), np.stack([lse[b, h].cpu().numpy() for b, h in units])[None], o_ref, lse_ref,
                "c4 full size")


def test_config5_full_size_prefix_and_tail():
    """c5 at full size (Hq64 Hkv8 N32768 d128 causal): prefix rows vs the oracle, tail rows vs float64."""
    torch = _torch()
    import odf_b200
    import oracle

    B, Hq, Hkv, N, D = 1, 64, 8, 32768, 128
    g = torch.Generator(device="cuda").manual_seed(55)
    q = torch.randn((B, Hq, N, D), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, Hkv, N, D), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, Hkv, N, D), generator=g, device="cuda").to(torch.bfloat16)
    o, lse = odf_b200.flash_fwd(q, k, v, causal=True, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    # causal rows < R only see keys < R: the prefix problem is exact for them
    R = 640
    heads = [0, 9, 63]
    qs = q[:, heads, :R].float().cpu().numpy()
    ks = k[:, [h // 8 for h in heads], :R].float().cpu().numpy()
    vs = v[:, [h // 8 for h in heads], :R].float().cpu().numpy()
    o_ref, lse_ref = oracle.flash_fwd(qs, ks, vs, causal=True)
    check_close(o[:, heads, :R].float().cpu().numpy(), lse[:, heads, :R].cpu().numpy(), o_ref, lse_ref,
                "c5 prefix")
    rows = [N - 129, N - 128, N - 1]
    for h in (5, 62):
        qh, kh, vh = q[0, h].float().cpu().numpy(), k[0, h // 8].float().cpu().numpy(), v[0, h // 8].float().cpu().numpy()
        o64, lse64 = _dense_rows_f64(qh, kh, vh, rows, causal=True, scale=1 / math.sqrt(D))
        assert np.abs(o[0, h, rows].float().cpu().numpy() - o64).max() <= O_MAX_ABS
        assert np.abs(lse[0, h, rows].cpu().numpy() - lse64).max() <= LSE_MAX_ABS


# --------------------------------------------------------------------------- work-item schedule
@pytest.mark.parametrize("causal", [False, True])
def test_greedy_blocked_schedule_matches_fixed_order(causal):
    """With a workspace and K/V beyond one ~32 MB block, the plain d=128 kernel hands items out
    greedily in blocks of (batch, kv-head) units (here 8 + a partial block of 3); without one it
    uses the fixed snake order.  Every item is computed the same way, so the two are bit-identical;
    rows of the prefix are also checked against the oracle."""
    import ctypes as C

    import odf_b200

    torch = _torch()
    B, Hq, Hk, N, D = 1, 22, 11, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn((B, h, N, D), generator=g, device="cuda").to(torch.bfloat16) for h in (Hq, Hk, Hk))
    o_dyn, lse_dyn = odf_b200.flash_fwd(q, k, v, causal=causal, out_dtype=torch.bfloat16)
    o_fix = torch.empty_like(o_dyn)
    lse_fix = torch.empty_like(lse_dyn)
    p, keep = odf_b200.fill_params(q, k, v, o_fix, lse_fix, causal=causal, scale=1.0 / math.sqrt(D),
                                   block_mask=None, mask_block=(128, 128), alibi=False, alibi_slopes_host=None,
                                   softcap=0.0, workspace=None, visits=None)
    lib = odf_b200.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.odf_flash_fwd_sm100(C.byref(p), C.c_void_p(stream)) == 0, odf_b200.last_error()
    torch.cuda.synchronize()
    assert torch.equal(o_dyn, o_fix)
    assert torch.equal(lse_dyn, lse_fix)
    if causal:  # causal prefix rows depend only on the key prefix: check them against the oracle
        R = 384
        qh, kh, vh = (x[:, :, :R].float().cpu().numpy() for x in (q, k, v))
        o_ref, lse_ref = oracle_fwd(qh, kh, vh, causal=True)
        check_close(o_dyn[:, :, :R].float().cpu().numpy(), lse_dyn[:, :, :R].cpu().numpy(), o_ref, lse_ref,
                    "greedy schedule prefix")
    assert odf_b200.device_status() == 0


# --------------------------------------------------------------------------- same-shape bias
def _bias(seed, shape, scale=2.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("case", ["full_gqa_causal", "head_broadcast", "key_row_softcap", "strided_keys",
                                  "query_col", "mask", "d64_softcap"])
def test_same_shape_bias(case):
    """BiasKind::SameShapeTile (qk_score_tile.cpp:28-47): s*scale + bias[b,h,qi,kj] (then soft-cap),
    with broadcast and strided bias layouts, against the oracle (itself pinned to the reference's
    ScoreBiasFn path)."""
    torch = _torch()
    import oracle

    B, H, Hk, M, N, D = 2, 4, 2, 300, 300, 128
    kw, okw = {}, {}
    if case == "full_gqa_causal":
        bias = _bias(1, (B, H, M, N))
        kw["causal"] = okw["causal"] = True
    elif case == "head_broadcast":
        bias = _bias(2, (1, 1, M, N))
    elif case == "key_row_softcap":
        bias = _bias(3, (1, 1, 1, N))
        kw["causal"] = okw["causal"] = True
        kw["softcap"] = okw["softcap"] = 30.0
    elif case == "strided_keys":  # bias[..., ::2] of a wider tensor: key stride 2 (scalar path)
        wide = _bias(4, (B, H, M, 2 * N))
        bias = wide[..., ::2]
    elif case == "query_col":
        bias = _bias(5, (B, 1, M, 1))
        kw["causal"] = okw["causal"] = True
    elif case == "mask":
        bias = _bias(6, (1, H, M, N))
        mask = oracle.sliding_window_prefix_mask(3, 1, 1)
        kw.update(causal=True, block_mask=mask, mask_block=(128, 128))
        okw.update(causal=True, mask=mask, mask_block=(128, 128))
    else:  # d64_softcap
        D = 64
        bias = _bias(7, (B, H, M, N))
        kw["softcap"] = okw["softcap"] = 20.0
    q, k, v = make_qkv(30, B, H, Hk, M, N, D)
    if case == "strided_keys":
        dev_bias = to_dev(wide, torch.float32)[..., ::2]
        assert dev_bias.stride(3) == 2
    else:
        dev_bias = to_dev(bias, torch.float32)
    o, lse = run_gpu(q, k, v, bias=dev_bias, **kw)
    o_ref, lse_ref = oracle_fwd(q, k, v, bias=bias, **okw)
    check_close(o, lse, o_ref, lse_ref, f"bias {case}")


def test_same_shape_bias_host_entry():
    """The host entry stages each (batch, head) bias plane (or one broadcast plane) per chunk and
    equals the device entry on the same values."""
    import odf_b200

    B, H, Hk, M, N, D = 2, 8, 2, 257, 333, 128
    q, k, v = make_qkv(31, B, H, Hk, M, N, D)
    for bias in (_bias(8, (B, H, M, N)), _bias(9, (1, 1, M, N)), _bias(10, (1, 1, 1, N))):
        lse = np.empty((B, H, M), dtype=np.float32)
        o, _ = odf_b200.flash_fwd_host(q, k, v, causal=True, bias=bias, lse_out=lse)
        o_dev, lse_dev = run_gpu(q, k, v, causal=True, bias=to_dev(bias, _torch().float32))
        assert np.array_equal(o, o_dev)
        assert np.array_equal(lse, lse_dev)
        o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, bias=bias)
        check_close(o, lse, o_ref, lse_ref, "bias host entry")


# --------------------------------------------------------------------------- host entry / status
@pytest.mark.parametrize("in_dtype", ["f32", "bf16"])
def test_host_entry_matches_device_entry(in_dtype):
    """odf_flash_fwd_host (host buffers, fp32 or bf16) equals the device entry on the same values."""
    import odf_b200
    import oracle

    H, Hk = 8, 2
    q, k, v = make_qkv(16, 2, H, Hk, 333, 333, 128)
    lse = np.empty((2, H, 333), dtype=np.float32)
    if in_dtype == "f32":
        hq, hk, hv = q, k, v
    else:
        hq, hk, hv = (np.ascontiguousarray((x.view(np.uint32) >> 16).astype(np.uint16)) for x in (q, k, v))
    o, _ = odf_b200.flash_fwd_host(hq, hk, hv, causal=True, alibi=True, lse_out=lse)
    o_dev, lse_dev = run_gpu(q, k, v, causal=True, alibi=True)
    assert np.array_equal(o, o_dev)
    assert np.array_equal(lse, lse_dev)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, alibi_slopes=oracle.alibi_slopes(H))
    check_close(o, lse, o_ref, lse_ref, "host entry")


@pytest.mark.parametrize("n_tiles,spike_tile", [(48, 1), (48, 30), (48, 47), (16, 9), (16, 15)])
def test_running_max_jump_on_long_key_range(n_tiles, spike_tile):
    """16 or more KV tiles (the variant that takes the exponentials against the running max before
    checking it): one K tile scaled by 8 lifts its scores far above the running max, so rows whose
    max moves past 2^8 are recomputed with the max pass; O and LSE still match the oracle."""
    q, k, v = make_qkv(51 + spike_tile + n_tiles, 1, 2, 2, 256, n_tiles * 128, 128)
    k[:, :, spike_tile * 128:(spike_tile + 1) * 128, :] *= 8.0  # a power of two: still bf16 values
    o, lse = run_gpu(q, k, v)
    o_ref, lse_ref = oracle_fwd(q, k, v)
    check_close(o, lse, o_ref, lse_ref, f"spike in tile {spike_tile}")


@pytest.mark.parametrize("mod,in_dtype", [("alibi", "bf16"), ("head_key_bias", "bf16"), ("alibi", "f32")])
def test_host_entry_split_first_and_last_units(mod, in_dtype):
    """A problem large enough for four or more host chunks (B 1, 32 q-heads over 8 kv-heads,
    N 8192): the first and last kv-head units are split into query-head sub-chunks, whose
    per-head ALiBi slopes and bias planes are shifted to their heads, and fp32 inputs are
    converted per sub-chunk; the result equals the device entry bit for bit."""
    import odf_b200

    B, H, Hk, N, D = 1, 32, 8, 8192, 128
    rng = np.random.default_rng(41)
    q, k, v = (np.ascontiguousarray((rng.standard_normal((B, h, N, D)).astype(np.float32).view(np.uint32) >> 16)
                                    .astype(np.uint16)) for h in (H, Hk, Hk))
    if in_dtype == "f32":  # the same bf16 values, given as fp32 (converted exactly on the device)
        hq, hk, hv = ((x.astype(np.uint32) << 16).view(np.float32) for x in (q, k, v))
    else:
        hq, hk, hv = q, k, v
    kw, dkw = {}, {}
    if mod == "alibi":
        kw["alibi"] = dkw["alibi"] = True
    elif mod == "block_mask":
        import oracle

        mask = oracle.sliding_window_prefix_mask(N // 128, 6, 3)
        kw.update(block_mask=mask, mask_block=(128, 128))
        dkw.update(block_mask=mask, mask_block=(128, 128))
    else:
        bias = rng.standard_normal((1, H, 1, N)).astype(np.float32)
        kw["bias"], dkw["bias"] = bias, to_dev(bias, _torch().float32)
    lse = np.empty((B, H, N), dtype=np.float32)
    o, _ = odf_b200.flash_fwd_host(hq, hk, hv, causal=True, lse_out=lse, **kw)
    torch = _torch()
    tq, tk, tv = (torch.from_numpy(x.astype(np.int16)).view(torch.bfloat16).cuda() for x in (q, k, v))
    o_dev = torch.empty((B, H, N, D), dtype=torch.float32, device="cuda")
    lse_dev = torch.empty((B, H, N), dtype=torch.float32, device="cuda")
    odf_b200.flash_fwd(tq, tk, tv, causal=True, out=o_dev, lse_out=lse_dev, **dkw)
    torch.cuda.synchronize()
    assert np.array_equal(o, o_dev.cpu().numpy())
    assert np.array_equal(lse, lse_dev.cpu().numpy())


def test_invalid_arguments_raise_before_launch():
    torch = _torch()
    import odf_b200

    q = torch.zeros((1, 3, 64, 64), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((1, 2, 64, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        odf_b200.flash_fwd(q, k, k)  # 3 q-heads over 2 kv-heads
    q96 = torch.zeros((1, 1, 64, 96), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(odf_b200.OdfError) as e:
        odf_b200.flash_fwd(q96, q96, q96)
    assert e.value.code == odf_b200.ODF_ERR_UNSUPPORTED


def test_device_status_clean_after_runs():
    """No bounded in-kernel wait ever gave up during the suite."""
    import odf_b200

    assert odf_b200.device_status(clear=True) == 0


@pytest.mark.parametrize("mod,in_dtype", [("alibi", "bf16"), ("head_key_bias", "f32"), ("block_mask", "bf16")])
def test_host_entry_few_units_in_query_head_pieces(mod, in_dtype):
    """Fewer than four (batch, kv-head) units (here 2 units of 8 query heads, N 9600): the host
    entry cuts each unit into pieces of query heads that share one upload of the unit's K/V (the
    shape one GPU gets when a GQA problem is split over several GPUs).  Per-piece ALiBi slopes,
    bias planes and fp32 conversion included, the result equals the device entry bit for bit."""
    import odf_b200

    B, H, Hk, N, D = 1, 16, 2, 9600, 128
    rng = np.random.default_rng(43)
    q, k, v = (np.ascontiguousarray((rng.standard_normal((B, h, N, D)).astype(np.float32).view(np.uint32) >> 16)
                                    .astype(np.uint16)) for h in (H, Hk, Hk))
    if in_dtype == "f32":
        hq, hk, hv = ((x.astype(np.uint32) << 16).view(np.float32) for x in (q, k, v))
    else:
        hq, hk, hv = q, k, v
    kw, dkw = {}, {}
    if mod == "alibi":
        kw["alibi"] = dkw["alibi"] = True
    elif mod == "block_mask":
        import oracle

        mask = oracle.sliding_window_prefix_mask(N // 128, 6, 3)
        kw.update(block_mask=mask, mask_block=(128, 128))
        dkw.update(block_mask=mask, mask_block=(128, 128))
    else:
        bias = rng.standard_normal((1, H, 1, N)).astype(np.float32)
        kw["bias"], dkw["bias"] = bias, to_dev(bias, _torch().float32)
    lse = np.empty((B, H, N), dtype=np.float32)
    o, _ = odf_b200.flash_fwd_host(hq, hk, hv, causal=True, lse_out=lse, **kw)
    torch = _torch()
    tq, tk, tv = (torch.from_numpy(x.astype(np.int16)).view(torch.bfloat16).cuda() for x in (q, k, v))
    o_dev = torch.empty((B, H, N, D), dtype=torch.float32, device="cuda")
    lse_dev = torch.empty((B, H, N), dtype=torch.float32, device="cuda")
    odf_b200.flash_fwd(tq, tk, tv, causal=True, out=o_dev, lse_out=lse_dev, **dkw)
    torch.cuda.synchronize()
    assert np.array_equal(o, o_dev.cpu().numpy())
    assert np.array_equal(lse, lse_dev.cpu().numpy())


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("mod", ["none", "alibi", "softcap", "alibi_softcap", "bias", "bias_softcap"])
@pytest.mark.parametrize("masked", [False, True])
def test_variant_matrix_gqa_ragged(d, causal, mod, masked):
    """Every kernel instantiation (d, score mod) crossed with causal / non-causal and with a block
    mask whose blocks do not line up with the 128x128 tiles, on GQA (4 q-heads over 2 kv-heads)
    with M != N and ragged tile ends, against the oracle."""
    import oracle

    torch = _torch()
    B, H, Hk, M, N = 1, 4, 2, 200, 330
    q, k, v = make_qkv(200 + d + 7 * causal + 3 * masked, B, H, Hk, M, N, d, scale=1.3)
    kw, okw = {"causal": causal}, {"causal": causal}
    if "alibi" in mod:
        kw["alibi"] = True
        okw["alibi_slopes"] = oracle.alibi_slopes(H)
    if "softcap" in mod:
        kw["softcap"] = okw["softcap"] = 7.5
    if mod.startswith("bias"):
        bias = _bias(60 + d, (1, H, M, N), scale=1.5)
        kw["bias"] = to_dev(bias, torch.float32)
        okw["bias"] = bias
    if masked:
        rng = np.random.default_rng(61 + d)
        mb = (48, 80)
        mask = (rng.random((-(-M // mb[0]), -(-N // mb[1]))) > 0.3).astype(np.uint8)
        mask[:, 0] = 1  # every query block sees at least one key block
        kw.update(block_mask=mask, mask_block=mb)
        okw.update(mask=mask, mask_block=mb)
    o, lse = run_gpu(q, k, v, **kw)
    o_ref, lse_ref = oracle_fwd(q, k, v, **okw)
    check_close(o, lse, o_ref, lse_ref, f"d={d} causal={causal} {mod} masked={masked}")


@pytest.mark.parametrize("m", [1, 16, 300])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("want_lse", [True, False])
def test_few_query_rows_long_keys(m, causal, want_lse):
    """Decode- and prefill-shaped problems: a few query rows against 8192 keys (GQA 8 over 2, d=128),
    which run the long-range variant (64 KV tiles) with one partial query tile; causal stays
    top-left aligned (row qi sees keys 0..qi).  O (and LSE when asked for) against the oracle;
    without an LSE buffer the kernel writes none."""
    q, k, v = make_qkv(300 + m + 2 * causal, 1, 8, 2, m, 8192, 128)
    o, lse = run_gpu(q, k, v, causal=causal, want_lse=want_lse)
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=causal)
    assert (lse is None) == (not want_lse)
    check_close(o, lse, o_ref, lse_ref if want_lse else None, f"m={m} causal={causal}")


# --------------------------------------------------------------------------- KV splits
def _splits_of(q, k, v, **kw):
    """Workspace bytes the launch asks for beyond the 256-byte counter (> 0: it splits its keys)."""
    import ctypes as C

    import odf_b200

    torch = _torch()
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    o = torch.empty(qd.shape[:3] + (vd.shape[3],), dtype=torch.float32, device="cuda")
    lse = torch.empty(qd.shape[:3], dtype=torch.float32, device="cuda")
    p, keep = odf_b200.fill_params(qd, kd, vd, o, lse, causal=kw.get("causal", False),
                                   scale=1.0 / math.sqrt(q.shape[3]), block_mask=None, mask_block=(128, 128),
                                   alibi=kw.get("alibi", False), alibi_slopes_host=None,
                                   softcap=kw.get("softcap", 0.0), workspace=None, visits=None)
    return odf_b200.load_library().odf_fwd_workspace_size(C.byref(p)) - 256


def _run_without_workspace(q, k, v, **kw):
    """The same launch through the C ABI without a workspace: no KV splits, fixed order."""
    import ctypes as C

    import odf_b200

    torch = _torch()
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    o = torch.empty(qd.shape[:3] + (vd.shape[3],), dtype=torch.float32, device="cuda")
    lse = torch.empty(qd.shape[:3], dtype=torch.float32, device="cuda")
    p, keep = odf_b200.fill_params(qd, kd, vd, o, lse, causal=kw.get("causal", False),
                                   scale=1.0 / math.sqrt(q.shape[3]), block_mask=None, mask_block=(128, 128),
                                   alibi=kw.get("alibi", False), alibi_slopes_host=None,
                                   softcap=kw.get("softcap", 0.0), workspace=None, visits=None,
                                   bias=kw.get("bias"))
    lib = odf_b200.load_library()
    assert lib.odf_flash_fwd_sm100(C.byref(p), C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0, \
        odf_b200.last_error()
    torch.cuda.synchronize()
    return o.cpu().numpy(), lse.cpu().numpy()


KV_SPLIT_CASES = {
    # (B, Hq, Hkv, M, N, D, kwargs): few query tiles over long key ranges, the shapes whose items
    # would leave most SMs idle without splits
    "decode_dense_d128_ragged": (1, 2, 1, 64, 3000, 128, {}),
    "decode_dense_d64": (1, 3, 3, 1, 4096, 64, {}),
    "causal_d64_later_splits_empty": (1, 2, 2, 200, 2500, 64, {"causal": True}),
    "causal_d128_square": (1, 1, 1, 1024, 1024, 128, {"causal": True}),
    "gqa_dense_d128": (1, 4, 1, 128, 4096, 128, {}),
    "alibi_softcap_dense_d128": (1, 3, 3, 130, 2100, 128, {"alibi": True, "softcap": 30.0}),
    "alibi_causal_d64": (1, 2, 2, 256, 2048, 64, {"alibi": True, "causal": True}),
    "softcap_causal_d128": (2, 1, 1, 300, 1900, 128, {"softcap": 15.0, "causal": True}),
}


@pytest.mark.parametrize("case", sorted(KV_SPLIT_CASES))
def test_kv_splits_vs_oracle(case):
    """Launches whose work items would leave more than half of the SMs idle cut each item's key
    range into splits (one item each), write normalised fp32 partials and merge them by their LSE.
    The merged O/LSE match the oracle, and the same launch without a workspace (no splits) agrees
    within the same tolerances; rows with no key in a split (causal) weigh it 0."""
    import oracle

    B, Hq, Hkv, M, N, D, kw = KV_SPLIT_CASES[case]
    q, k, v = make_qkv(40 + len(case), B, Hq, Hkv, M, N, D, scale=0.7)
    assert _splits_of(q, k, v, **kw) > 0, "this shape should split its key range"
    o, lse = run_gpu(q, k, v, **kw)
    okw = {"causal": kw.get("causal", False), "softcap": kw.get("softcap", 0.0)}
    if kw.get("alibi"):
        okw["alibi_slopes"] = oracle.alibi_slopes(Hq)
    o_ref, lse_ref = oracle_fwd(q, k, v, **okw)
    check_close(o, lse, o_ref, lse_ref, f"kv splits {case}")
    o_one, lse_one = _run_without_workspace(q, k, v, **kw)
    check_close(o_one, lse_one, o_ref, lse_ref, f"no splits {case}")


def test_kv_splits_same_shape_bias():
    """A strided same-shape bias with KV splits (key offsets of later splits) against the oracle."""
    B, H, M, N, D = 1, 2, 100, 1800, 128
    q, k, v = make_qkv(47, B, H, H, M, N, D)
    bias = _bias(11, (B, H, M, N))
    assert _splits_of(q, k, v, causal=True) > 0
    o, lse = run_gpu(q, k, v, causal=True, bias=to_dev(bias, _torch().float32))
    o_ref, lse_ref = oracle_fwd(q, k, v, causal=True, bias=bias)
    check_close(o, lse, o_ref, lse_ref, "kv splits bias")


@pytest.mark.parametrize("in_dtype", ["f32", "bf16"])
def test_kv_splits_host_entry_equals_device_entry(in_dtype):
    """The host entry's chunks split the key range as one device launch of the whole problem does,
    so the two results are equal bit for bit (and match the oracle)."""
    import odf_b200

    B, H, Hk, M, N, D = 1, 4, 2, 100, 3000, 128
    q, k, v = make_qkv(48, B, H, Hk, M, N, D)
    assert _splits_of(q, k, v) > 0
    if in_dtype == "f32":
        hq, hk, hv = q, k, v
    else:
        hq, hk, hv = (np.ascontiguousarray((x.view(np.uint32) >> 16).astype(np.uint16)) for x in (q, k, v))
    lse = np.empty((B, H, M), dtype=np.float32)
    o, _ = odf_b200.flash_fwd_host(hq, hk, hv, lse_out=lse)
    o_dev, lse_dev = run_gpu(q, k, v)
    assert np.array_equal(o, o_dev)
    assert np.array_equal(lse, lse_dev)
    o_ref, lse_ref = oracle_fwd(q, k, v)
    check_close(o, lse, o_ref, lse_ref, "kv splits host entry")


def test_kv_splits_fewer_when_workspace_is_smaller():
    """A workspace with room for fewer splits than the plan asks for: the launch splits as many ways
    as fit (here 3 instead of 6) and still matches the oracle."""
    import ctypes as C

    import odf_b200

    torch = _torch()
    B, H, Hk, M, N, D = 1, 2, 1, 64, 3000, 128
    q, k, v = make_qkv(49, B, H, Hk, M, N, D)
    up = lambda n: -(-n // 256) * 256
    full = _splits_of(q, k, v)
    assert full == up(6 * B * H * M * D * 4) + up(6 * B * H * M * 4)  # six splits of four KV tiles
    room = up(3 * B * H * M * D * 4) + up(3 * B * H * M * 4)
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    o = torch.empty((B, H, M, D), dtype=torch.float32, device="cuda")
    lse = torch.empty((B, H, M), dtype=torch.float32, device="cuda")
    ws = torch.zeros(256 + room, dtype=torch.uint8, device="cuda")
    p, keep = odf_b200.fill_params(qd, kd, vd, o, lse, causal=False, scale=1.0 / math.sqrt(D), block_mask=None,
                                   mask_block=(128, 128), alibi=False, alibi_slopes_host=None, softcap=0.0,
                                   workspace=None, visits=None)
    p.workspace = ws.data_ptr()
    p.workspace_bytes = 256 + room
    lib = odf_b200.load_library()
    assert lib.odf_flash_fwd_sm100(C.byref(p), C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0, \
        odf_b200.last_error()
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle_fwd(q, k, v)
    check_close(o.cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, "kv splits in a smaller workspace")
