"""bench.py's command line and its reference arm, on CPU.

The reference arm times the reference's own CPU path (the NumPy-backend
restatement of BASELINE config 2) and needs no GPU, so its JSON line is
checked here against the keys the round driver reads; the b200 arm needs a
B200 and is exercised by the GPU runs.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench(*args, timeout=240):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)


def _json_lines(out: str):
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    proc = _bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = _json_lines(proc.stdout)
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == "GEMV 16384x16384 + DOT 2^26 float32 HBM throughput"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_workloads_say_unavailable():
    proc = _bench("--impl", "reference", "--workload", "norm", "--steps", "1", "--warmup", "3")
    assert proc.returncode == 0, proc.stderr[-2000:]
    (d,) = _json_lines(proc.stdout)
    assert d["impl"] == "reference" and d["unavailable"]


def test_fewer_than_three_warmup_steps_are_rejected():
    proc = _bench("--impl", "reference", "--steps", "1", "--warmup", "2", timeout=60)
    assert proc.returncode == 2
    assert "--warmup must be >= 3" in proc.stderr
