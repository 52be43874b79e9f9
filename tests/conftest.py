"""Shared pytest setup: the `gpu` marker, import paths and seeded input helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for sub in ("oracle", "dnn-flash_b200"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA path through the C ABI")


def gpu_available() -> bool:
    try:
        import torch
    except ImportError:
        return False
    return torch.cuda.is_available()


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def make_qkv(seed, B, Hq, Hkv, M, N, D, DV=None, scale=1.0):
    """Seeded N(0,1)*scale inputs rounded to bf16, as fp32 numpy arrays [B,H,T,D]."""
    import oracle

    DV = D if DV is None else DV
    rng = np.random.default_rng(seed)
    q = oracle.round_bf16((rng.standard_normal((B, Hq, M, D)) * scale).astype(np.float32))
    k = oracle.round_bf16((rng.standard_normal((B, Hkv, N, D)) * scale).astype(np.float32))
    v = oracle.round_bf16((rng.standard_normal((B, Hkv, N, DV)) * scale).astype(np.float32))
    return q, k, v
