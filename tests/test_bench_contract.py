"""bench.py's JSON contract, checked on CPU through the reference arm (the
only arm that runs without a GPU): one JSON line with the metric, unit and
config of the B200 arm, the CPU baseline it measured and an e2e block."""

from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [line for line in run.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("MSDA fwd+bwd") and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1 and d["value"] > 0
    assert d["config"]["workload"].startswith("config 4")
    base = d["cpu_baseline"]
    assert base["value"] == d["value"] and base["kind"] in ("port", "reference") and base["cores"] >= 1
    assert base["sample"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["e2e"]["d2h_bytes_per_step"] == 0
