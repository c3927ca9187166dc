"""Launch settings change timing only: programmatic dependent launch on / off (SH_PDL), the GEMM tile order
(SH_GEMM_GROUP_M: 1 = row-major, default 8 = grouped), the pair tile width (SH_GEMM_PAIR_BN: 256 instead of the
planner's 512 for long K) and the barrier grouping of the 2-CTA kernel (SH_GEMM_KS=1: one barrier per stage instead
of one per stage pair) give bit-identical encoder and GEMM outputs. Each setting is read once per process, so
every variant runs in its own process (tests/launch_modes_worker.py)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _hashes(**env) -> str:
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "launch_modes_worker.py")], capture_output=True,
                       text=True, env=dict(os.environ, **env), timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("HASH ")]
    assert len(lines) == 1, r.stdout
    return lines[0]


def test_launch_modes_are_bit_identical():
    base = _hashes()
    assert _hashes(SH_PDL="0") == base
    assert _hashes(SH_GEMM_GROUP_M="1") == base
    assert _hashes(SH_GEMM_GROUP_M="3", SH_PDL="0") == base
    assert _hashes(SH_GEMM_PAIR_BN="256") == base
    assert _hashes(SH_GEMM_KS="1") == base
    assert _hashes(SH_GEMM_KS="1", SH_GEMM_PAIR_BN="256") == base
