"""The checked build (the library compiled with -DODF_CHECKED: in-kernel invariants on work-item
decode, KV entries, the tensor-memory base, ring loads issued vs waited, P.V counts vs softmax
tiles and the causal ALiBi bound) over problems that reach every scheduling and score-mod path
(KV splits included):
no invariant may fail, the status word stays clean, and the results match the oracle.  The
checked library runs in its own process (tests/checked_build_run.py)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
CHECKED = ROOT / "dnn-flash_b200" / "lib" / "libodf_sm100_checked.so"


def test_checked_build_invariants_hold():
    assert CHECKED.exists(), f"{CHECKED} is missing: build it with __graft_entry__.build()"
    proc = subprocess.run([sys.executable, str(ROOT / "tests" / "checked_build_run.py")], capture_output=True,
                          text=True, timeout=600, env=dict(os.environ))
    assert proc.returncode == 0, proc.stderr[-3000:]
    results = [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]
    assert len(results) == 12, proc.stdout[-2000:]
    for r in results:
        assert r["rc"] == 0 and r["check_bits"] == 0 and r["status"] == 0, r
        assert r["o_rel_l2"] <= 1e-2 and r["o_max_abs"] <= 2e-2 and r["lse_max_abs"] <= 1e-3, r
        assert r["lse_inf_pattern"], r


def test_shipped_library_has_no_checks():
    import ctypes as C

    import odf_b200

    bits = C.c_uint32(7)
    assert odf_b200.load_library().odf_debug_check_bits(C.byref(bits)) == odf_b200.ODF_ERR_UNSUPPORTED
