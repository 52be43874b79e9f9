"""The C++ API (include/onednn_flash/*.hpp) as a drop-in for the reference's.

* CPU: every planner function (make_score_mod_plan, make_block_mask_plan,
  make_causal_mask_tile_descriptor, make_runtime_plan, make_runtime_plan_cache_key,
  backend_name, tile_kernel_name) returns exactly what the reference's own code
  (oracle/_ref, built from its sources) returns, over a grid of inputs.
* GPU: each attention entry point (standard_attention, flash_attention_tiled,
  flash_attention_q_tile, flash_attention_qk_pv_tile, flash_attention_qk_pv_tile_ws,
  flash_attention_batched_qk_pv_tile, run_attention) on host vectors/pointers and,
  for the raw-pointer ones, on device pointers, against the reference's outputs at
  the parity tolerances; error behaviour keeps the reference's exception types.
"""
from __future__ import annotations

import shutil
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import ROOT, make_qkv

O_REL_L2 = 1e-2
O_MAX_ABS = 2e-2
LSE_MAX_ABS = 1e-3


@pytest.fixture(scope="session")
def driver(tmp_path_factory):
    lib_dir = ROOT / "dnn-flash_b200" / "lib"
    if not (lib_dir / "libodf_sm100.so").exists():
        pytest.skip("libodf_sm100.so not built")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = tmp_path_factory.mktemp("cppdrv") / "cpp_api_check"
    cmd = [nvcc, "-std=c++17", "-O2", "-Wno-deprecated-gpu-targets", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "cpp" / "cpp_api_check.cpp"), "-o", str(out), f"-L{lib_dir}", "-lodf_sm100",
           "-Xlinker", "-rpath", "-Xlinker", str(lib_dir)]
    subprocess.run(cmd, check=True, capture_output=True)
    return out


needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference build (oracle/_ref) not present")


@needs_ref
def test_planner_matches_reference(driver):
    out = subprocess.run([str(driver), "planner"], check=True, capture_output=True, text=True).stdout.splitlines()
    counts = {"SMP": 0, "BMP": 0, "CMT": 0, "RTP": 0, "BKN": 0, "TKN": 0}
    for line in out:
        head, _, rest = line.partition("|")
        tag, *args = head.split()
        if tag == "SMP":
            kind, dtype, has_scale, bias, post = map(int, args)
            assert rest == oracle.ref_score_mod_plan(kind, dtype, has_scale, 0.125, bias, post), line
        elif tag == "BMP":
            kind, ql, kl = map(int, args)
            assert rest == oracle.ref_block_mask_plan(kind, ql, kl), line
        elif tag == "CMT":
            assert rest == oracle.ref_causal_mask_tile(*map(int, args)), line
        elif tag == "RTP":
            ints = list(map(int, args))
            ref = oracle.ref_runtime_plan(ints[:17], 0.25, ints[17], ints[18]).replace("\n", "\\n")
            assert rest == ref, line
        elif tag == "BKN":
            assert rest == oracle.ref_backend_name(int(args[0]))
        elif tag == "TKN":
            assert rest == oracle.ref_tile_kernel_name(int(args[0]))
        else:
            continue
        counts[tag] += 1
    assert counts["SMP"] == 360 and counts["RTP"] == 30720 and counts["BMP"] == 27 and counts["CMT"] == 36


def test_sm100_plan_describes_the_gpu_kernel(driver):
    out = subprocess.run([str(driver), "planner"], check=True, capture_output=True, text=True).stdout.splitlines()
    gpu = [ln for ln in out if ln.startswith("GPU|")][0].split("|")  # GPU|<signature with |>|fallback|backend
    assert gpu[-2] == "none" and gpu[-1] == "sm100_tcgen05"
    sig = "|".join(gpu[1:-2])
    assert "scale_additive_bias:alibi_generated:bf16:softcap" in sig and "|causal|" in sig
    gpu96 = [ln for ln in out if ln.startswith("GPU96|")][0].split("|")
    assert gpu96[1] == "unsupported_shape" and gpu96[2] == "reference"


# ---------------------------------------------------------------------------------- GPU cases
APIS = {"standard": 0, "tiled": 1, "q_tile": 2, "qk_pv_tile": 3, "ws": 4, "batched": 5, "run_standard": 6,
        "run_tiled": 7}


def run_api(driver, tmp_path, api, q, k, v, *, causal=False, scale=None, q_block=16, k_block=32, mask=None,
            mask_block=(1, 1), slopes=None, softcap=0.0, want_lse=True, device=False, bias=None):
    B, H, M, D = q.shape
    _, Hkv, N, _ = k.shape
    DV = v.shape[3]
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    hdr = [APIS[api], B, H, Hkv, M, N, D, DV, int(causal), q_block, k_block, mask_block[0], mask_block[1],
           mask.shape[0] if mask is not None else 0, mask.shape[1] if mask is not None else 0,
           1 if slopes is not None else (2 if bias is not None else 0)]
    inp = tmp_path / f"{api}_in.bin"
    outp = tmp_path / f"{api}_out.bin"
    with open(inp, "wb") as f:
        f.write(struct.pack("<16i", *hdr))
        f.write(struct.pack("<4f", scale, softcap, float(want_lse), float(device)))
        for t in (q, k, v):
            f.write(np.ascontiguousarray(t, dtype=np.float32).tobytes())
        if mask is not None:
            f.write(np.ascontiguousarray(mask, dtype=np.uint8).tobytes())
        if slopes is not None:
            f.write(np.asarray(slopes, dtype=np.float32).tobytes())
        elif bias is not None:
            f.write(np.ascontiguousarray(np.broadcast_to(bias, (B, H, M, N)), dtype=np.float32).tobytes())
    proc = subprocess.run([str(driver), "run", str(inp), str(outp)], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr
    raw = np.fromfile(outp, dtype=np.uint8)
    status = struct.unpack("<i", raw[:4].tobytes())[0]
    body = np.frombuffer(raw[4:].tobytes(), dtype=np.float32)
    o = body[: B * H * M * DV].reshape(B, H, M, DV)
    lse = body[B * H * M * DV:].reshape(B, H, M)
    return status, o, lse, proc.stderr


def close(o, lse, o_ref, lse_ref=None):
    diff = o.astype(np.float64) - o_ref.astype(np.float64)
    assert np.linalg.norm(diff) / max(np.linalg.norm(o_ref), 1e-30) <= O_REL_L2
    assert np.abs(diff).max() <= O_MAX_ABS
    if lse_ref is not None:
        fin = np.isfinite(lse_ref)
        assert np.abs(lse[fin] - lse_ref[fin]).max() <= LSE_MAX_ABS


@pytest.mark.gpu
@pytest.mark.parametrize("api", ["standard", "tiled", "q_tile", "qk_pv_tile", "run_standard", "run_tiled"])
def test_vector_entry_points_match_reference(driver, tmp_path, api):
    q, k, v = make_qkv(60, 1, 1, 1, 300, 300, 64)
    status, o, lse, err = run_api(driver, tmp_path, api, q, k, v, causal=True)
    assert status == 0, err
    ref_variant = {"standard": "standard", "run_standard": "standard"}.get(api, "tiled" if "tiled" in api else api)
    r = oracle.ref_fwd(ref_variant, q, k, v, causal=True, q_block=16, k_block=32)
    _, lse_ref = oracle.flash_fwd(q, k, v, causal=True)
    close(o, lse, r, lse_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("device", [False, True])
def test_workspace_entry_with_block_mask_and_alibi(driver, tmp_path, device):
    q, k, v = make_qkv(61, 1, 1, 1, 520, 520, 128)
    mask = oracle.sliding_window_prefix_mask(9, 3, 2)
    slopes = np.array([0.0625], dtype=np.float32)
    status, o, lse, err = run_api(driver, tmp_path, "ws", q, k, v, causal=True, mask=mask, mask_block=(64, 64),
                                  slopes=slopes, device=device)
    assert status == 0, err
    r = oracle.ref_fwd("flash_ws", q, k, v, causal=True, q_block=16, k_block=32, mask=mask, mask_block=(64, 64),
                       alibi_slopes=slopes)
    _, lse_ref = oracle.flash_fwd(q, k, v, causal=True, mask=mask, mask_block=(64, 64), alibi_slopes=slopes)
    close(o, lse, r, lse_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("device", [False, True])
def test_batched_entry_point_gqa_softcap(driver, tmp_path, device):
    q, k, v = make_qkv(62, 2, 8, 2, 384, 384, 128)
    status, o, lse, err = run_api(driver, tmp_path, "batched", q, k, v, causal=True, softcap=30.0, device=device)
    assert status == 0, err
    o_ref, lse_ref = oracle.flash_fwd(q, k, v, causal=True, softcap=30.0)
    close(o, lse, o_ref, lse_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("device", [False, True])
@pytest.mark.parametrize("api", ["ws", "batched"])
def test_same_shape_bias_through_cpp_api(driver, tmp_path, device, api):
    """AttentionOptions{bias_kind = SameShapeTile, bias} on host and device pointers, against the
    oracle (equal to the reference's ScoreBiasFn path bit for bit, test_oracle_vs_reference.py)."""
    B, H = (1, 1) if api == "ws" else (2, 4)
    q, k, v = make_qkv(66, B, H, H, 270, 300, 128)
    bias = (np.random.default_rng(67).standard_normal((B, H, 270, 300)) * 2.0).astype(np.float32)
    status, o, lse, err = run_api(driver, tmp_path, api, q, k, v, causal=True, bias=bias, device=device)
    assert status == 0, err
    r, lse_ref = oracle.flash_fwd(q, k, v, causal=True, q_block=16, k_block=32, bias=bias)
    close(o, lse, r, lse_ref)


@pytest.mark.gpu
def test_batched_matches_reference_batched_driver(driver, tmp_path):
    """flash_attention_batched_qk_pv_tile vs the reference's own batched driver (as shipped)."""
    q, k, v = make_qkv(63, 2, 3, 3, 200, 200, 64)
    status, o, _, err = run_api(driver, tmp_path, "batched", q, k, v, causal=True, want_lse=False)
    assert status == 0, err
    r = oracle.ref_fwd("batched", q, k, v, causal=True, q_block=16, k_block=32)
    close(o, None, r)


@pytest.mark.gpu
def test_errors_keep_reference_exception_types(driver, tmp_path):
    q, k, v = make_qkv(64, 1, 1, 1, 64, 64, 64)
    status, _, _, err = run_api(driver, tmp_path, "tiled", q, k, v, k_block=0)
    assert status == 1 and "key_block_size must be non-zero" in err      # std::invalid_argument
    status, _, _, err = run_api(driver, tmp_path, "q_tile", q, k, v, q_block=0)
    assert status == 1 and "query_block_size must be non-zero" in err
    q96, k96, v96 = make_qkv(65, 1, 1, 1, 64, 64, 96)
    status, _, _, err = run_api(driver, tmp_path, "standard", q96, k96, v96)
    assert status == 2 and "head_dim" in err                             # std::runtime_error (unsupported)
    bad_mask = np.ones((2, 2), dtype=np.uint8)
    status, _, _, err = run_api(driver, tmp_path, "ws", q, k, v, mask=bad_mask, mask_block=(0, 32))
    assert status == 1 and "BlockMask block sizes must be non-zero" in err
