"""bench.py's reference arm on the CPU: one JSON line with the metric, unit and config of the GPU arm, `impl:
reference`, a `cpu_baseline` describing the run and an `e2e` without host copies (the contract the round-end driver
reads). The GPU arm needs a B200 and is exercised by the GPU runs."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "encoder images/s" and d["unit"] == "images/s"
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 0 and d["value"] > 0
    assert d["config"]["workload"].startswith("SigLIP-base 12-layer encoder")
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] in ("port", "reference")
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"] and d["cpu_baseline"]["blas"]
    assert d["e2e"] == {"value": d["value"], "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_roofline_traffic_comes_from_the_committed_profile():
    b = _bench_module()
    t = b.profile_traffic("gemm_fc1_m131072")        # the default workload's FC1 launch (B = 512 x S = 256 rows)
    assert t is not None and 0.5e9 < t < 2e9
    assert b.profile_traffic("no_such_kernel") is None


def test_clock_summary_reads_nvml_samples():
    b = _bench_module()
    c = b.ClockSampler(0)
    c.nvml = type("FakeNvml", (), {"nvmlShutdown": staticmethod(lambda: None)})
    c.thread = type("T", (), {"join": lambda self, timeout=None: None})()
    c.samples = [(1965.0, 1965.0, 0)]                 # before the timed region: dropped by mark()
    c.mark()
    c.samples += [(1400.0, 1965.0, 0x4), (1420.0, 1965.0, 0x4), (1380.0, 1965.0, 0x4 | 0x40)]
    got = c.stop()
    assert got["sm_mhz"] == 1400.0 and got["sm_max_mhz"] == 1965.0 and got["samples"] == 3
    assert got["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
