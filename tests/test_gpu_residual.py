"""The compiled plans' residual b - A @ x on the GPU (pb_gemv_residual) and
the lowering's elementwise groups.

The residual is one GEMV launch with the subtraction in its epilogue; the
product is rounded to the dtype before the subtraction, as in the eager
expression (src/openpacho/_gemv.py:1-6), so the result must carry exactly
the bits of the unfused pair pb_gemv + elementwise subtract, and meet the GEMV
bound (plus one rounding of the difference) against the NumPy-backend oracle.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

import front as pb
from oracle import numpy_backend, tolerance
from pacho_b200.lowering import B200Lowering

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 3), (1000, 1), (513, 4097), (16384, 16384),
                                       (3, 200000), (40000, 64), (5, 0)])
def test_residual_matches_unfused_pair_bit_for_bit(b200, dtype, rows, cols):
    rng = np.random.default_rng(rows * 31 + cols)
    A = rng.uniform(-1, 1, (rows, cols)).astype(dtype)
    x = rng.uniform(-1, 1, cols).astype(dtype)
    b = rng.uniform(-1, 1, rows).astype(dtype)
    if rows > 3 and cols > 3:
        A[1, 2], b[2], b[3] = np.inf, np.nan, -0.0
    dA, dx, db = (pb.asarray(v, backend=b200) for v in (A, x, b))
    fused = pb.wrap(b200.residual_matvec(dA, dx, db), (rows,), dtype, b200).numpy()
    unfused = (db - dA @ dx).numpy()
    assert fused.tobytes() == unfused.tobytes()
    with np.errstate(all="ignore"):
        y = numpy_backend.matmul(A, x)
        want = numpy_backend.elementwise("subtract", (b, y), dtype)
    finite = np.isfinite(want)
    assert np.array_equal(np.isnan(fused), np.isnan(want))
    assert np.array_equal(fused[np.isinf(want)], want[np.isinf(want)])
    bound = tolerance.gemm_bound(A, x) + tolerance.unit_roundoff(dtype) * (
        np.abs(b.astype(np.float64)) + np.abs(y.astype(np.float64)))
    err = np.abs(fused.astype(np.float64) - want.astype(np.float64))
    assert np.all(err[finite] <= 2 * bound[finite])


def test_residual_rejects_mismatched_operands(b200):
    A = pb.asarray(np.ones((4, 3), np.float32), backend=b200)
    x = pb.asarray(np.ones(3, np.float32), backend=b200)
    with pytest.raises(ValueError):
        b200.residual_matvec(A, x, pb.asarray(np.ones(5, np.float32), backend=b200))
    with pytest.raises(ValueError):
        b200.residual_matvec(A, x, pb.asarray(np.ones(4, np.float64), backend=b200))


def _node(op, inputs, resolved, shape, dtype):
    return SimpleNamespace(op=op, inputs=inputs, resolved=tuple(np.dtype(t) for t in resolved),
                           shape=shape, dtype=np.dtype(dtype), attrs={})


def test_lowering_runs_an_elementwise_group_step_by_step(b200):
    """(b * 2.0 - x).astype(float64) + b as a compiled group: each step in its
    own dtype, inputs cast to the resolved dtypes first -- the NumPy bits."""
    rng = np.random.default_rng(3)
    b = rng.standard_normal(1000).astype(np.float32)
    x = rng.standard_normal(1000).astype(np.float32)
    lb, lx = _node("input", (), (), (1000,), np.float32), _node("input", (), (), (1000,), np.float32)
    two = _node("scalar", (), (), (), np.float32)
    mul = _node("multiply", (lb, two), (np.float32, np.float32, np.float32), (1000,), np.float32)
    sub = _node("subtract", (mul, lx), (np.float32, np.float32, np.float32), (1000,), np.float32)
    cast = _node("cast", (sub,), (np.float32, np.float64), (1000,), np.float64)
    add = _node("add", (cast, lb), (np.float64, np.float64, np.float64), (1000,), np.float64)
    lowering = B200Lowering(b200)
    args, payload = lowering.prepare_fused(add, [mul, sub, cast, add], [lb, two, lx])
    scalar = pb.Scalar(2.0, np.float32)
    data = lowering.run_fused(add, payload, args, [pb.asarray(b, backend=b200), scalar,
                                                   pb.asarray(x, backend=b200)])
    got = pb.wrap(data, (1000,), np.float64, b200).numpy()
    want = (b * np.float32(2.0) - x).astype(np.float64) + b.astype(np.float64)
    assert got.tobytes() == want.tobytes()
