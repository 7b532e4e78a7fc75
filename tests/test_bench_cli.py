"""bench.py's command line and JSON contract, on the CPU.

The reference arm (``--impl reference``) times the reference's float64 host
evaluation and needs no GPU, so it runs here: one JSON line on stdout with
the contract's keys, the metric BASELINE.json names, and an end-to-end record
with no host/device traffic.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def run_bench(*args: str, timeout: int = 300) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    done = run_bench("--impl", "reference", "--workload", "add", "--steps", "2", "--warmup", "1", "--only")
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [line for line in done.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, lines
    rec = json.loads(lines[0])
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert rec["metric"] == baseline["metric"]
    assert rec["impl"] == "reference"
    for key in ("value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["steps"] == 2 and rec["warmup"] == 1 and rec["n_gpus"] == 1
    assert rec["value"] > 0 and rec["unit"] == "GB/s" and rec["higher_is_better"] is True
    assert rec["e2e"]["value"] == rec["value"]
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["e2e"]["d2h_bytes_per_step"] == 0
    assert rec["cpu_baseline"]["kind"] == "port" and rec["cpu_baseline"]["cores"] >= 1
    assert rec["config"]["workload"]


def test_help_lists_the_options():
    done = run_bench("--help", timeout=120)
    assert done.returncode == 0, done.stderr[-2000:]
    for flag in ("--gpus", "--steps", "--warmup", "--workload", "--impl", "--only", "--no-graph", "--shard-of"):
        assert flag in done.stdout, flag
