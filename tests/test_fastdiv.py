"""The multiply-shift division by launch constants (Granlund-Montgomery) that
the GEMM tile schedules and batch maps use, checked on the host against plain
integer division: tests/fastdiv_check.cu, built with nvcc as host code."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_fast_division_matches_plain_division(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    exe = tmp_path / "fastdiv_check"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
                    "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-I",
                    str(ROOT / "open-pacho_b200" / "csrc"), str(ROOT / "tests" / "fastdiv_check.cu"),
                    "-o", str(exe)], check=True, capture_output=True, text=True)
    proc = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "mismatches 0" in proc.stdout
