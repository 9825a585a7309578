"""bench.py's JSON contract on the CPU: the reference arm (the reference's round on the host cores)
prints one line with the contract's keys, and the workload helpers behave."""

import json
import subprocess
import sys
from pathlib import Path

import bench

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == "verify rounds/sec" and d["value"] > 0
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] in ("port", "reference")
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "qwen3-4b-b16"


def test_workload_prompt_lengths():
    assert bench.prompt_len(bench.WORKLOADS["qwen3-4b-b16"], 5) == 2048
    lens = [bench.prompt_len(bench.WORKLOADS["qwen3-8b-b64"], r) for r in range(8)]
    assert all(1024 <= x <= 8192 for x in lens) and len(set(lens)) > 1
    assert lens == [bench.prompt_len(bench.WORKLOADS["qwen3-8b-b64"], r) for r in range(8)]  # seeded


def test_clock_summary_uses_samples_of_the_timed_region():
    import datetime

    def row(t, sm, *reasons):
        ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        act = ["Active" if r else "Not Active" for r in reasons]
        return f"{ts}, 0, {sm}, 1965, 900.0, 0x0, {act[0]}, {act[1]}, {act[2]}, {act[3]}"

    t0 = 1_800_000_000.0
    lines = [row(t0 - 1.0, 800, 0, 0, 0, 0),            # idle, before the region
             row(t0 + 0.01, 1965, 0, 0, 0, 1), row(t0 + 0.03, 1950, 0, 0, 0, 1),
             row(t0 + 2.0, 700, 1, 0, 0, 0), "garbage"]   # after it
    d = bench.summarize_clocks(lines, t0, t0 + 0.04, 0.02)
    assert d["samples_in_region"] == 2 and d["sm_mhz"] == 1957.5 and d["sm_max_mhz"] == 1965.0
    assert d["reasons"] == ["sw_power_cap"]
    # no sample inside: the nearest one stands in
    d = bench.summarize_clocks(lines[:1], t0, t0 + 0.04, 0.02)
    assert d["samples_in_region"] == 0 and d["sm_mhz"] == 800
    assert bench.summarize_clocks([], t0, t0, 0.02)["reasons"] == ["no samples"]


def test_clock_summary_without_readable_timestamps_uses_every_sample():
    lines = ["Tue Dec 1 00:00:00 2026, 0, 1900, 1965, 800.0, 0x0, Not Active, Not Active, Not Active, Active",
             "Tue Dec 1 00:00:01 2026, 0, 1800, 1965, 800.0, 0x0, Not Active, Not Active, Not Active, Not Active"]
    d = bench.summarize_clocks(lines, 0.0, 1.0, 0.02)
    assert d["sm_mhz"] == 1850 and d["reasons"] == ["sw_power_cap"] and d["samples"] == 2
