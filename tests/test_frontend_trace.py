"""The recorded front-end trace reproduces OpenPacho's NumPy backend (CPU).

tests/golden/make_frontend_trace.py ran programs through OpenPacho's own front
end with b200 registered (the recording host stand-in computing each backend
call with the NumPy-backend oracle) and, separately, on OpenPacho's NumPy
backend.  The program outputs the recorded calls produced must equal the
NumPy backend's bit for bit: then the recorded calls are exactly the work the
front end asks of b200, and tests/test_gpu_frontend_replay.py checks each of
them on the GPU.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def trace():
    return (json.loads((GOLDEN / "frontend_trace.json").read_text()),
            np.load(GOLDEN / "frontend_trace.npz"))


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    if a.dtype.kind == "f":
        return np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(
            a[~np.isnan(a)].view(np.uint8), b[~np.isnan(b)].view(np.uint8))
    return np.array_equal(a, b)


def test_trace_outputs_equal_the_numpy_backend(trace):
    meta, values = trace
    assert len(meta["programs"]) >= 8
    for prog in meta["programs"]:
        for k, out in enumerate(prog["outputs"]):
            got = values[f"b{out['buf']}"].reshape(out["shape"])
            want = values[f"final/{prog['program']}/{k}"]
            assert _same(got, want), (prog["program"], k)


def test_trace_covers_the_protocol(trace):
    meta, _ = trace
    methods = {c["method"] for c in meta["calls"]}
    assert {"upload", "matmul", "norm", "elementwise", "reduce", "gather", "residual_matvec",
            "download", "full"} <= methods
    programs = {c["program"] for c in meta["calls"]}
    assert "conjugate_gradient" in programs and "compiled_residual" in programs
