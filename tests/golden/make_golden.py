"""Generate tests/golden/reference_cases.npz from the REFERENCE itself.

Run in a checkout where the reference is present (it is not needed afterwards):

    python tests/golden/make_golden.py [reference_dir]

For every case the inputs are seeded N(0,1) values rounded to bf16 (stored as
uint16 bf16 bits), and the outputs come from:
  * ref_ws:   the reference's C++ flash_attention_qk_pv_tile_ws
              (src/onednn_flash/attention.cpp:486-695), through oracle/_ref, which is
              compiled from the reference's unmodified sources;
  * ref_np:   the reference's numpy golden model flash_attention_reference
              (python/onednn_flash/reference.py:91-156), imported from the checkout.
The ALiBi bias is passed to both as the reference's own score_bias functor
slope * (kj - qi).
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "oracle"))

import oracle  # noqa: E402

# name: (B, Hq, Hkv, M, N, D, causal, q_block, k_block, mask_kind, mask_block, alibi)
CASES = {
    "dense_d64": (1, 2, 2, 192, 192, 64, False, 16, 32, None, None, False),
    "causal_ragged": (1, 2, 2, 200, 170, 64, True, 16, 32, None, None, False),
    "m_lt_n": (1, 1, 1, 100, 260, 64, False, 32, 64, None, None, False),
    "gqa_d128": (1, 4, 2, 136, 136, 128, True, 16, 32, None, None, False),
    "blockmask_alibi": (1, 2, 2, 260, 260, 64, True, 16, 32, "diag_random", (64, 64), True),
    "tiles128": (1, 1, 1, 384, 384, 128, True, 128, 128, None, None, False),
}


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def make_mask(kind, M, N, block, rng):
    if kind is None:
        return None
    nq, nk = -(-M // block[0]), -(-N // block[1])
    mask = (rng.random((nq, nk)) > 0.4).astype(np.uint8)
    for i in range(min(nq, nk)):
        mask[i, i] = 1  # every row keeps its diagonal block, so no row is fully masked
    return mask


def load_numpy_reference(ref_dir: Path):
    spec = importlib.util.spec_from_file_location("odf_reference_numpy",
                                                  ref_dir / "python" / "onednn_flash" / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ref_dir = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ODF_REFERENCE_DIR", "/root/reference"))
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref is not built (run __graft_entry__.build() with the reference present)")
    npref = load_numpy_reference(ref_dir)
    out = {}
    for idx, (name, (B, Hq, Hkv, M, N, D, causal, qb, kb, mkind, mblock, alibi)) in enumerate(CASES.items()):
        rng = np.random.default_rng(1000 + idx)
        q = oracle.round_bf16(rng.standard_normal((B, Hq, M, D)).astype(np.float32))
        k = oracle.round_bf16(rng.standard_normal((B, Hkv, N, D)).astype(np.float32))
        v = oracle.round_bf16(rng.standard_normal((B, Hkv, N, D)).astype(np.float32))
        mask = make_mask(mkind, M, N, mblock, rng)
        slopes = oracle.alibi_slopes(Hq) if alibi else None
        kw = dict(causal=causal, q_block=qb, k_block=kb, alibi_slopes=slopes)
        if mask is not None:
            kw.update(mask=mask, mask_block=mblock)
        ref_ws = oracle.ref_fwd("flash_ws", q, k, v, **kw)
        ref_np = np.zeros_like(ref_ws)
        group = Hq // Hkv
        for b in range(B):
            for h in range(Hq):
                bias = None
                if alibi:
                    s = float(slopes[h])
                    bias = (lambda qi, kj, s=s: np.float32(s) * np.float32(kj - qi))
                ref_np[b, h] = npref.flash_attention_reference(
                    q[b, h], k[b, h // group], v[b, h // group], scale=1.0 / np.sqrt(D), causal=causal,
                    key_block_size=kb, block_mask=mask, query_block_size=mblock[0] if mask is not None else 1,
                    block_mask_key_block_size=mblock[1] if mask is not None else None, score_bias=bias)
        prefix = f"{name}__"
        out[prefix + "q"] = bf16_bits(q)
        out[prefix + "k"] = bf16_bits(k)
        out[prefix + "v"] = bf16_bits(v)
        out[prefix + "ref_ws"] = ref_ws
        out[prefix + "ref_np"] = ref_np.astype(np.float32)
        out[prefix + "meta"] = np.array([B, Hq, Hkv, M, N, D, int(causal), qb, kb,
                                         mblock[0] if mask is not None else 0, mblock[1] if mask is not None else 0,
                                         int(alibi)], dtype=np.int64)
        if mask is not None:
            out[prefix + "mask"] = mask
        print(f"{name}: ws vs numpy max diff {np.abs(ref_ws - ref_np).max():.2e}")
    np.savez_compressed(HERE / "reference_cases.npz", **out)
    print(f"wrote {HERE / 'reference_cases.npz'}")


if __name__ == "__main__":
    main()
