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
