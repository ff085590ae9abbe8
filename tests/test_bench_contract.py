"""bench.py's command line and its reference arm, on CPU.

The reference arm times the reference's own CPU path (the NumPy-backend
restatement of every BASELINE config) and needs no GPU, so its JSON line is
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


def _check_record(d, unit=None):
    assert d["value"] > 0 and d["unit"] in ("GB/s", "TFLOP/s")
    if unit:
        assert d["unit"] == unit
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith(("BASELINE config", "x @ A", "b - A @ x"))


def test_reference_arm_prints_one_contract_line_for_the_suite():
    """Headline config 3 plus one sub-record per other config, every one timed
    through the NumPy-backend restatement with the config the b200 arm prints."""
    proc = _bench("--impl", "reference", "--steps", "1", "--warmup", "3", timeout=900)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = _json_lines(proc.stdout)
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == "batched broadcast GEMM (8,16,512,256)@(1,16,256,384) float32 TFLOP/s"
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    _check_record(d, "TFLOP/s")
    assert d["config"]["parallelism"] == "batch split x1 (B broadcast from rank 0 by NCCL)"
    names = set(d["configs"])
    assert {"config1_gemm_f32_1024", "config2_gemv_dot_f32", "config4a_norm_f32", "config4a_norm_f64",
            "config4b_rows_f32", "config4b_rows_f64", "config5_gemm_f32_16384",
            "config5_gemm_f64_8192"} <= names
    for rec in d["configs"].values():
        _check_record(rec)


def test_reference_arm_single_workload():
    proc = _bench("--impl", "reference", "--workload", "norm", "--steps", "1", "--warmup", "3")
    assert proc.returncode == 0, proc.stderr[-2000:]
    (d,) = _json_lines(proc.stdout)
    assert d["impl"] == "reference" and d["metric"] == "scaled norm full 2^28 float32 GB/s"
    _check_record(d, "GB/s")
    assert "configs" not in d


def test_reference_arm_uses_every_core_under_torchrun_thread_limits():
    """torchrun exports OMP_NUM_THREADS=1; the reference arm still runs
    OpenBLAS on every core this process may use."""
    import os

    env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload",
                           "gemm1024", "--steps", "1", "--warmup", "3"], cwd=ROOT, capture_output=True,
                          text=True, timeout=240, env=env)
    assert proc.returncode == 0, proc.stderr[-2000:]
    (d,) = _json_lines(proc.stdout)
    assert d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))


def test_fewer_than_three_warmup_steps_are_rejected():
    proc = _bench("--impl", "reference", "--steps", "1", "--warmup", "2", timeout=60)
    assert proc.returncode == 2
    assert "--warmup must be >= 3" in proc.stderr
