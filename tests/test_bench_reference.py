"""The bench's reference arm (`bench.py --impl reference`) on the CPU: one JSON line on the product
arm's metric, unit, direction and config (the same `config` object the product arm prints, so the
two lines describe the same workload), timing the CPU oracle the way the reference's own bench
times its CPU engine, with the keys the bench contract names (cpu_baseline, e2e without host
copies)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _reference_line(*extra):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "1",
                          *extra], capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def _common(d, metric, unit):
    assert d["impl"] == "reference"
    assert d["metric"] == metric
    assert d["unit"] == unit and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_decode_line(full_model_path):
    d = _reference_line()
    _common(d, bench.DECODE_METRIC, "tok/s")
    assert d["config"] == bench.workload_config("ai130", 1)
    # timed like bench.rs: decode positions right after the real 130-id prompt
    assert "positions 130.." in d["cpu_baseline"]["sample"]


@pytest.mark.parametrize("cfg", ["prefill", "gemv"])
def test_reference_arm_other_configs(cfg, full_model_path):
    d = _reference_line("--config", cfg)
    if cfg == "prefill":
        _common(d, bench.PREFILL_METRIC, "tok/s")
        assert "positions 0.." in d["cpu_baseline"]["sample"]
    else:
        _common(d, bench.GEMV_METRIC, "GB/s")
        assert set(d["shapes"]) == set(bench.GEMV_SHAPES)
    assert d["config"] == bench.workload_config(cfg, 1)


def test_workload_config_is_engine_free():
    for name in bench.CONFIGS:
        c = bench.workload_config(name, 4)
        assert c["workload"].startswith("configs[")
        assert "engine" not in c and "impl" not in c


def test_clock_summary_flags_throttle_reasons():
    """The clock record the bench line carries: median SM clock under load, the max clock, and every
    throttle reason seen active in any sample (nvidia-smi csv rows, as the sampler collects them)."""
    cs = bench.ClockSampler(0)
    cs.lines = [
        "0, 1965, 1965, 700.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1950, 1965, 980.2, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 990.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
    ]
    got = cs.summary()
    assert got["sm_mhz"] == 1965.0 and got["sm_max_mhz"] == 1965.0 and got["samples"] == 3
    assert got["reasons"] == ["sw_power_cap"]
    cs.lines = []
    assert cs.summary()["sm_mhz"] is None
