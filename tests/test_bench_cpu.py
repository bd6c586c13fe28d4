"""bench.py on the host: the clock-sampling summary that goes into every JSON line, and the reference arm (one run
of `--impl reference` prints exactly one JSON line with the keys the result collector reads: the same metric,
unit and direction as the GPU arm, a cpu_baseline describing the run, and an e2e object with zero copy bytes)."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def test_clock_summary_parses_sampled_rows():
    """The `clocks` object: median SM clock under load, the max clock, and every throttle reason seen Active
    (the nvidia-smi csv,noheader,nounits rows of the query bench.py issues; malformed rows are skipped)."""
    import bench
    c = bench.Clocks(0)
    rows = ["0, 1965, 1965, 640.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
            "0, 1800, 1965, 990.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
            "0, 1890, 1965, 985.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
            "[N/A] garbled line",
            "0, 1900, 1965, 700.0, 0x0000000000000000, Not Active, Not Active, Active, Not Active"]
    c.f.write("\n".join(rows) + "\n")
    s = c.summary()
    assert s["sm_mhz"] == 1895.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 4
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_clock_summary_without_samples():
    import bench
    c = bench.Clocks(0)
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ)
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(key, None)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == "TB/s" and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] >= 3 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
