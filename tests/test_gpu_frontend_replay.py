"""OpenPacho's front end over the real b200 kernels, by replaying its calls.

OpenPacho is not installed on the GPU machines, so the calls its front end
makes on b200 were recorded in the build container
(tests/golden/make_frontend_trace.py: ``matmul``/``@`` with broadcast batches
and ``padding=``, ``dot``, vector @ matrix, mixed dtypes, ``linalg.norm``
with axes and ``keepdims``, ``compile`` with this package's lowering -- fused
residual GEMVs, elementwise groups and their reductions --, casts, views,
means, and the reference's example conjugate-gradient solver).  Here every
recorded call runs on the B200 backend exactly as the front end made it
(method, shapes, dtypes, axes, strides, host scalars), with the recorded
values of its operands, and its output is checked against the recorded
NumPy-backend value: GEMM-like calls within 4*K*u*(|A||B|), norms within 8u,
correctly rounded elementwise operations, casts, gathers, fills and extrema
bit for bit, transcendental operations within 8u, sums within 4*n*u*sum|x|.
tests/test_frontend_trace.py pins the recorded values to OpenPacho's own
NumPy backend.
"""

from __future__ import annotations

import json
from math import prod
from pathlib import Path

import numpy as np
import pytest

import front
from oracle import numpy_backend, tolerance

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TRACE = json.loads((GOLDEN / "frontend_trace.json").read_text())
VALUES = np.load(GOLDEN / "frontend_trace.npz")
CORRECTLY_ROUNDED = {"add", "subtract", "multiply", "true_divide", "divide", "negative", "positive",
                     "absolute", "sqrt", "equal", "not_equal", "less", "less_equal", "greater",
                     "greater_equal", "isfinite", "cast", "where"}
COMPUTING = ("matmul", "norm", "elementwise", "gather", "reduce", "residual_matvec", "full")


def _value(ref):
    return VALUES[f"b{ref['buf']}"].reshape(ref["shape"])


def _same(got, want):
    if got.shape != want.shape or got.dtype != want.dtype:
        return False
    if want.dtype.kind != "f":
        return np.array_equal(got, want)
    return np.array_equal(np.isnan(got), np.isnan(want)) and np.array_equal(
        got[~np.isnan(want)].view(np.uint8), want[~np.isnan(want)].view(np.uint8))


def _operand(backend, ref, cache):
    if "scalar" in ref:
        return front.Scalar(ref["scalar"], ref["dtype"])
    key = ref["buf"], tuple(ref["shape"]), ref["dtype"]
    if key not in cache:
        cache[key] = front.asarray(_value(ref).astype(ref["dtype"]), backend=backend)
    return cache[key]


def _check(call, got, args):
    method = call["method"]
    want = VALUES[f"b{call['out']}"].reshape(got.shape)
    if method in ("gather", "full"):
        return _same(got, want)
    if method == "matmul":
        a, b = (_value(r) for r in call["args"])
        return tolerance.gemm_violations(got, want, a, b) == 0
    if method == "residual_matvec":
        A, x, b = (_value(r) for r in call["args"])
        y = numpy_backend.matmul(A, x)
        bound = tolerance.gemm_bound(A, x) + tolerance.unit_roundoff(A.dtype) * (
            np.abs(b.astype(np.float64)) + np.abs(y.astype(np.float64)))
        fin = np.isfinite(want)
        return np.array_equal(np.isnan(got), np.isnan(want)) and bool(
            np.all(np.abs(got[fin].astype(np.float64) - want[fin]) <= 2 * bound[fin]))
    if method == "norm":
        x = _value(call["args"][0])
        exact = numpy_backend.norm_data(x.astype(np.float64), tuple(call["axes"]), np.float64)
        return tolerance.norm_violations(got.reshape(-1), want.reshape(-1), dtype=want.dtype,
                                         exact=exact) == 0
    if method == "reduce":
        if call["operation"] != "sum":
            return _same(got, want)
        x = _value(call["args"][0])
        axes = tuple(call["axes"])
        n = max(1, prod(x.shape[i] for i in axes))
        u = tolerance.unit_roundoff(want.dtype) if want.dtype.kind == "f" else 0.0
        bound = 4 * n * u * np.sum(np.abs(x.astype(np.float64)), axis=axes).reshape(-1)
        return bool(np.all(np.abs(got.reshape(-1).astype(np.float64) - want.reshape(-1)) <= bound))
    if method == "elementwise":
        if call["name"] in CORRECTLY_ROUNDED or want.dtype.kind == "b":
            return _same(got, want)
        fin = np.isfinite(want)
        u = tolerance.unit_roundoff(want.dtype)
        return np.array_equal(np.isnan(got), np.isnan(want)) and bool(np.all(
            np.abs(got[fin].astype(np.float64) - want[fin]) <= 8 * u * np.abs(want[fin].astype(np.float64))
            + np.finfo(want.dtype).tiny))
    raise AssertionError(method)


def _run(backend, call, cache):
    method = call["method"]
    args = [_operand(backend, r, cache) for r in call.get("args", [])]
    if method == "matmul":
        data = backend.matmul(*args, tuple(call["shape"]), call["dtype"])
        shape, dtype = call["shape"], call["dtype"]
    elif method == "norm":
        data = backend.norm(args[0], tuple(call["axes"]), call["keepdims"], call["dtype"])
        x = args[0]
        shape = [d for i, d in enumerate(x.shape) if i not in call["axes"]]
        dtype = call["dtype"]
    elif method == "elementwise":
        data = backend.elementwise(call["name"], args, tuple(call["shape"]), call["dtype"])
        shape, dtype = call["shape"], call["dtype"]
    elif method == "gather":
        data = backend.gather(args[0], tuple(call["shape"]), call["offset"], tuple(call["strides"]))
        shape, dtype = call["shape"], args[0].dtype
    elif method == "reduce":
        data = backend.reduce(args[0], tuple(call["axes"]), call["keepdims"], call["dtype"],
                              operation=call["operation"])
        x = args[0]
        shape = [d for i, d in enumerate(x.shape) if i not in call["axes"]]
        dtype = call["dtype"]
    elif method == "residual_matvec":
        data = backend.residual_matvec(*args)
        shape, dtype = [args[0].shape[0]], args[0].dtype
    else:  # full
        data = backend.full(tuple(call["shape"]), call["value"], call["dtype"])
        shape, dtype = call["shape"], call["dtype"]
    return front.wrap(data, shape, dtype, backend).numpy(), args


@pytest.mark.parametrize("program", [p["program"] for p in TRACE["programs"]])
def test_every_recorded_call_on_the_gpu(b200, program):
    calls = [c for c in TRACE["calls"] if c["program"] == program and c["method"] in COMPUTING]
    assert calls
    cache = {}
    bad = []
    for i, call in enumerate(calls):
        got, args = _run(b200, call, cache)
        if not _check(call, got, args):
            bad.append((i, call["method"], call.get("name"), call.get("shape")))
    assert not bad, bad
