"""The reference arm of bench.py (the CPU restatement on the host cores) runs
without a GPU: one short invocation, its JSON line checked for the fields
the measurement contract asks for."""
from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_line():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"]


def test_bench_cli_parses():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True,
                         text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0 and "--impl" in res.stdout and "--case" in res.stdout
