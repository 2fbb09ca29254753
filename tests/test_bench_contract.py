"""bench.py's output contract on the CPU: the reference arm's line and the
clock summary that goes into every timed line."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_reference_arm_prints_one_unavailable_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"],
                         capture_output=True, text=True, timeout=120, env={**os.environ, "RANK": "0"})
    assert out.returncode == 0, out.stderr
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"] and "metric" in d


def test_clock_summary_median_under_load_and_reasons():
    import bench
    rows = [
        "0, 1965, 1965, 120.5, 0x0, Not Active, Not Active, Not Active, Not Active",   # idle
        "0, 1800, 1965, 950.0, 0x4, Not Active, Not Active, Not Active, Active",       # power cap
        "0, 1900, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1950, 1965, 910.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage",
    ]
    s = bench.ClockSampler.summarize(rows)
    assert s["sm_mhz"] == 1900 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 4 and s["samples_under_load"] == 3
    thermal = bench.ClockSampler.summarize(
        ["0, 1400, 1965, 990.0, 0x40, Not Active, Active, Not Active, Not Active"])
    assert thermal["reasons"] == ["hw_thermal_slowdown"]
    assert bench.ClockSampler.summarize([])["sm_mhz"] is None
