"""Seeded random problems through both C-ABI entries against the CPU oracle.

Each case draws its shape and options from a fixed seed: batch, kv-heads and GQA group,
M and N (ragged, M != N), head_dim 64/128, causal or not, a score_mod (none, generated or
explicit ALiBi slopes -- some steep enough that causal d = 128 leaves out far tiles -- soft-cap,
both, a broadcast or full same-shape bias tensor), sometimes a block mask with block sizes
unrelated to the 128 x 128 tiles, bf16 or fp32 O, and the device entry
(odf_flash_fwd_sm100) or the host entry (odf_flash_fwd_host, fp32 or bf16 host inputs).
Tolerances as in test_flash_gpu.py, plus half a bf16 ulp of the value (2^-9 |O|) on bf16
outputs, whose rounding alone exceeds 2e-2 above |O| = 8.  The draws are deterministic, so a
failure names a case that reproduces.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import make_qkv

pytestmark = pytest.mark.gpu

O_REL_L2 = 1e-2
O_MAX_ABS = 2e-2
LSE_MAX_ABS = 1e-3
N_CASES = 120


def _case(i):
    rng = np.random.default_rng(1000 + i)
    c = {
        "B": int(rng.integers(1, 3)),
        "Hkv": int(rng.integers(1, 4)),
        "G": int(rng.choice([1, 2, 4])),
        "M": int(rng.integers(1, 700)),
        "N": int(rng.integers(1, 700)),
        "D": int(rng.choice([64, 128])),
        "causal": bool(rng.random() < 0.6),
        "mod": str(rng.choice(["none", "alibi", "alibi_steep", "softcap", "alibi_softcap", "bias_bcast",
                               "bias_full"])),
        "mask": bool(rng.random() < 0.25),
        "out_bf16": bool(rng.random() < 0.5),
        "entry": str(rng.choice(["device", "host_f32", "host_bf16"])),
        "in_scale": float(rng.choice([0.5, 1.0, 1.5])),
        "softcap": float(rng.choice([5.0, 20.0, 50.0])),
        "seed": int(rng.integers(0, 2 ** 31)),
    }
    if c["mask"]:
        c["mask_block"] = (int(rng.choice([32, 64, 128, 200])), int(rng.choice([48, 64, 128, 256])))
    return c


def _check(o, lse, o_ref, lse_ref, what, bf16_out):
    assert np.all(np.isfinite(o)), f"{what}: non-finite output"
    diff = o.astype(np.float64) - o_ref.astype(np.float64)
    rel = np.linalg.norm(diff) / max(np.linalg.norm(o_ref.astype(np.float64)), 1e-30)
    assert rel <= O_REL_L2, f"{what}: O rel-L2 {rel:.3e}"
    excess = np.abs(diff) - (O_MAX_ABS + (2.0 ** -9 * np.abs(o_ref) if bf16_out else 0.0))
    assert excess.max() <= 0.0, f"{what}: O max-abs {np.abs(diff).max():.3e}"
    fin = np.isfinite(lse_ref)
    assert np.array_equal(np.isfinite(lse), fin), f"{what}: LSE -inf pattern differs"
    if fin.any():
        e = np.abs(lse[fin] - lse_ref[fin]).max()
        assert e <= LSE_MAX_ABS, f"{what}: LSE max-abs {e:.3e}"


@pytest.mark.parametrize("i", range(N_CASES))
def test_random_problem_vs_oracle(i):
    import odf_b200
    import oracle
    import torch

    c = _case(i)
    B, Hkv, G, M, N, D = c["B"], c["Hkv"], c["G"], c["M"], c["N"], c["D"]
    Hq = Hkv * G
    what = f"case {i}: {c}"
    q, k, v = make_qkv(c["seed"] % 100000, B, Hq, Hkv, M, N, D, scale=c["in_scale"])
    rng = np.random.default_rng(c["seed"])
    alibi, slopes, softcap, bias = False, None, 0.0, None
    if c["mod"] in ("alibi", "alibi_softcap"):
        alibi = True
        if rng.random() < 0.5:
            slopes = rng.uniform(0.0, 1.0, Hq).astype(np.float32)
    elif c["mod"] == "alibi_steep":
        alibi, slopes = True, rng.choice([0.0, 0.25, 1.0, 4.0], Hq).astype(np.float32)
    if c["mod"] in ("softcap", "alibi_softcap"):
        softcap = c["softcap"]
    if c["mod"] == "bias_bcast":
        bias = rng.standard_normal((1, 1, M, N)).astype(np.float32)
    elif c["mod"] == "bias_full":
        bias = rng.standard_normal((B, Hq, M, N)).astype(np.float32)
    mask, mb = None, (128, 128)
    if c["mask"]:
        mb = c["mask_block"]
        mask = (rng.random((-(-M // mb[0]), -(-N // mb[1]))) > 0.3).astype(np.uint8)

    okw = dict(causal=c["causal"], softcap=softcap, mask=mask, mask_block=mb, bias=bias,
               alibi_slopes=(slopes if slopes is not None else oracle.alibi_slopes(Hq)) if alibi else None)
    o_ref, lse_ref = oracle.flash_fwd(q, k, v, **okw)

    kw = dict(causal=c["causal"], alibi=alibi, alibi_slopes=slopes, softcap=softcap, block_mask=mask, mask_block=mb)
    lse = np.empty((B, Hq, M), dtype=np.float32)
    if c["entry"] == "device":
        dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(torch.bfloat16)
        o_t, lse_t = odf_b200.flash_fwd(dev(q), dev(k), dev(v), out_dtype=torch.bfloat16 if c["out_bf16"] else None,
                                        bias=torch.from_numpy(bias).cuda() if bias is not None else None, **kw)
        torch.cuda.synchronize()
        o, lse = o_t.float().cpu().numpy(), lse_t.cpu().numpy()
    else:
        if c["entry"] == "host_f32":
            hq, hk, hv = q, k, v
        else:
            hq, hk, hv = (np.ascontiguousarray((x.view(np.uint32) >> 16).astype(np.uint16)) for x in (q, k, v))
        out = np.empty((B, Hq, M, D), dtype=np.uint16 if c["out_bf16"] else np.float32)
        odf_b200.flash_fwd_host(hq, hk, hv, out=out, lse_out=lse, bias=bias, **kw)
        o = (out.astype(np.uint32) << 16).view(np.float32) if c["out_bf16"] else out
    _check(o, lse, o_ref, lse_ref, what, c["out_bf16"])


def test_cases_cover_every_option():
    """The fixed draws reach every score_mod, both head dims, both entries' kinds and the mask."""
    cases = [_case(i) for i in range(N_CASES)]
    assert {c["mod"] for c in cases} == {"none", "alibi", "alibi_steep", "softcap", "alibi_softcap", "bias_bcast",
                                         "bias_full"}
    assert {c["D"] for c in cases} == {64, 128}
    assert {c["entry"] for c in cases} == {"device", "host_f32", "host_bf16"}
    assert any(c["mask"] for c in cases) and any(c["causal"] for c in cases)
    assert any(c["mod"] == "alibi_steep" and c["causal"] and c["D"] == 128 and not c["mask"] for c in cases)
