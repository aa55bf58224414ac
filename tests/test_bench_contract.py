"""bench.py's JSON line: every key the driver reads, with values that agree
with one another.  The reference arm (the oracle port on the host cores) runs
here on a small row sample; our arm needs the GPU."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

CONTRACT = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
            "scaling", "vs_baseline", "dtype", "data", "config", "e2e")


def run_bench(*args: str, timeout: int) -> dict:
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def check_common(line: dict, steps: int, warmup: int) -> None:
    for k in CONTRACT:
        assert k in line, k
    assert line["steps"] == steps and line["warmup"] == warmup and line["n_gpus"] == 1
    assert line["value"] > 0 and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["scaling"] in ("weak", "strong")
    assert line["vs_baseline"] is None  # BASELINE publishes no number for this metric
    assert "workload" in line["config"] and "model" not in line["config"]
    for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"):
        assert k in line["e2e"], k


def test_reference_arm_line():
    line = run_bench("--impl", "reference", "--steps", "3", "--warmup", "3", timeout=600)
    check_common(line, 3, 3)
    assert line["impl"] == "reference"
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["config"]["rows_per_step"] == 16384  # the benchmark's own config, whole passes


@pytest.mark.gpu
def test_our_arm_line():
    line = run_bench("--steps", "5", "--warmup", "3", "--no-extras", timeout=600)
    check_common(line, 5, 3)
    assert "impl" not in line
    roof = line["roofline"]
    assert roof["bound"] == "hbm" and roof["unit"] == "GB/s" and roof["peak"] > 0
    assert abs(roof["frac"] - roof["achieved"] / roof["peak"]) < 1e-3
    # a kernel that reads well above the copy peak is not doing its work
    assert 0.3 < roof["frac"] < 1.2
    e2e = line["e2e"]
    assert e2e["h2d_bytes_per_step"] == 16384 * 12288 * 8
    assert e2e["d2h_bytes_per_step"] == 16384 * (12288 + 192 * 4)
    assert 0 < e2e["value"] < line["value"]
    link = e2e["link"]
    assert link["h2d_gbs"] > 0 and link["d2h_gbs"] > 0
    assert 0 < link["frac"] <= 1.2  # the copies alone cannot be much slower than copies + kernel
    assert line["gpu_launches"] == 5
    v = line["verified"]
    assert v["mismatches"] == 0 and v["codes"] == 16384 * 12288 and v["scales"] == 16384 * 192
    assert e2e["outputs_match_device"] is True
    clk = line["clocks"]
    assert "sm_mhz" in clk and "reasons" in clk
    assert clk["samples"] >= 1  # readings taken while the queued timed region runs


def test_clock_summary_tolerates_missing_readings():
    """The clock record keeps the SM clock and throttle reasons when the
    driver does not give the memory clock, power or temperature, and counts
    only the samples inside the marked timed region."""
    import bench
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.ok, c.max_mhz, c.mem_max_mhz, c.period = True, 1965, None, 0.001
    # (host time, sm MHz, reasons, memory MHz, board W, GPU C)
    c.samples = [(0.5, 1000, 0x40, None, 100.0, 30), (1.0, 1965, 0x0, None, 700.0, None),
                 (1.5, 1950, 0x4, 3996, None, 55), (2.0, 1965, 0x0, 3996, 690.0, 40), (9.0, 900, 0x8, None, None, None)]
    c.t0, c.t1 = 0.9, 2.1
    s = c.summary()
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    assert s["mem_mhz"] == 3996 and s["power_w"] == 695.0 and s["temp_c_max"] == 55
    assert s["samples"] == 3
