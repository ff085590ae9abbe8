"""Elementwise, gather and reduce on the GPU against the NumPy-backend oracle.

These are the operations around the path (src/openpacho/backends.py:109-136,
src/openpacho/_cuda.py:416-492): astype, solver arithmetic, sum/mean/min/max,
transpose/diag.  Correctly rounded operations (+ - * / sqrt, sign changes,
comparisons, casts, where) must match bit for bit, NaN and signed zeros
included; exp/log/sin/cos/tanh/power within 4 ulp (8u relative).  Ends with a
conjugate-gradient solve through the public API, the downstream check the
reference's examples/solvers.py provides.
"""

from __future__ import annotations

import numpy as np
import pytest

import front as pb
from oracle import numpy_backend, tolerance

pytestmark = pytest.mark.gpu

EXACT = ("add", "subtract", "multiply", "true_divide", "negative", "positive", "absolute", "sqrt",
         "equal", "not_equal", "less", "less_equal", "greater", "greater_equal", "isfinite")
TRANSCENDENTAL = ("exp", "log", "sin", "cos", "tanh", "power")
BINARY = ("add", "subtract", "multiply", "true_divide", "power", "equal", "not_equal", "less",
          "less_equal", "greater", "greater_equal")


def _values(rng, shape, dtype):
    x = (rng.standard_normal(shape) * 4).astype(dtype)
    flat = x.reshape(-1)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0, 1e-30, 3.0], dtype)
    flat[: min(flat.size, specials.size)] = specials[: flat.size]
    return x


def _same(got, want):
    """Bit-for-bit equality, NaN matching NaN and the sign of zero kept."""
    assert got.shape == want.shape and got.dtype == want.dtype
    got, want = got.reshape(-1), want.reshape(-1)
    if want.dtype.kind == "b":
        return np.array_equal(got, want)
    return np.array_equal(got.view(np.uint8), want.view(np.uint8)) or (
        np.array_equal(np.isnan(got), np.isnan(want))
        and np.array_equal(got[~np.isnan(want)].view(np.uint8), want[~np.isnan(want)].view(np.uint8)))


def _close(got, want, dtype):
    u = tolerance.unit_roundoff(dtype)
    finite = np.isfinite(want)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])
    err = np.abs(got[finite].astype(np.float64) - want[finite].astype(np.float64))
    tiny = np.finfo(dtype).tiny
    assert np.all(err <= 8 * u * np.abs(want[finite].astype(np.float64)) + tiny)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("name", EXACT + TRANSCENDENTAL)
def test_ufuncs_match_oracle(b200, name, dtype):
    rng = np.random.default_rng(31)
    a = _values(rng, (3, 1, 257), dtype)
    b = _values(rng, (5, 1), dtype)  # broadcast against a: (3, 5, 257)
    if name == "power":
        a = np.abs(a)
    ufunc = getattr(np, name)
    inputs = (a, b) if name in BINARY else (a,)
    with np.errstate(all="ignore"):
        want = ufunc(*inputs)
    got = pb.asnumpy(ufunc(*(pb.asarray(x, backend=b200) for x in inputs)))
    if name in EXACT:
        assert _same(got, want), name
    else:
        _close(got, want, np.dtype(dtype))


def test_scalars_casts_where_and_bool(b200):
    rng = np.random.default_rng(32)
    x = _values(rng, (1000,), np.float32)
    dx = pb.asarray(x, backend=b200)
    with np.errstate(all="ignore"):
        assert _same(pb.asnumpy(dx * 2.5 - 1), x * np.float32(2.5) - np.float32(1))
        assert _same(pb.asnumpy(1 / dx), np.float32(1) / x)
    assert _same(pb.asnumpy(dx.astype(np.float64)), x.astype(np.float64))
    y = (rng.standard_normal(1000) * 1e40).astype(np.float64)  # overflows float32 to +-Inf
    with np.errstate(over="ignore"):
        want = y.astype(np.float32)
    assert _same(pb.asnumpy(pb.asarray(y, backend=b200).astype(np.float32)), want)
    mask = pb.asnumpy(pb.isfinite(dx))
    assert _same(mask, np.isfinite(x))
    assert _same(pb.asnumpy(pb.asarray(mask, backend=b200).astype(np.float32)), mask.astype(np.float32))
    assert _same(pb.asnumpy(dx.astype(np.bool_)), x.astype(np.bool_))
    sel = pb.asnumpy(pb.where(dx > 0, dx, 0.0))
    assert _same(sel, np.where(x > 0, x, np.float32(0)))
    assert _same(pb.asnumpy(pb.equal(pb.isfinite(dx), False)), np.equal(np.isfinite(x), False))
    z = pb.asnumpy(pb.zeros((3, 0), np.float32, backend=b200) + 1)
    assert z.shape == (3, 0)


@pytest.mark.parametrize("shape,axes", [((1 << 24,), (0,)), ((300, 5000), (1,)), ((300, 5000), (0,)),
                                        ((7, 9, 11, 13), (0, 2)), ((4, 3, 2), (0, 1, 2)),
                                        ((70000, 3), (1,)), ((5, 0, 3), (1,))])
@pytest.mark.parametrize("operation", ["sum", "min", "max"])
def test_reductions_match_oracle(b200, shape, axes, operation):
    if operation != "sum" and 0 in [shape[i] for i in axes]:
        pytest.skip("extrema of an empty set raise in the front end")
    rng = np.random.default_rng(33)
    x = rng.standard_normal(shape).astype(np.float32)
    if x.size:
        x.reshape(-1)[:: max(1, x.size // 7)] = -0.0
    dx = pb.asarray(x, backend=b200)
    data = b200.reduce(dx, axes, False, np.float32, operation=operation)
    kept = tuple(d for i, d in enumerate(shape) if i not in axes)
    got = pb.asnumpy(pb.wrap(data, kept, np.float32, b200))
    want = numpy_backend.reduce(x, axes, False, np.float32, operation)
    if operation == "sum":
        # |s - s_ref| <= 4 n u sum|x|, n the number of terms
        n = max(1, int(np.prod([shape[i] for i in axes])))
        bound = 4 * n * tolerance.unit_roundoff(np.float32) * np.sum(np.abs(x), axis=axes,
                                                                      dtype=np.float64)
        assert np.all(np.abs(got.astype(np.float64) - want) <= bound)
    else:
        assert _same(got, want)


def test_extrema_nan_signed_zero_bool_and_api(b200):
    x = np.array([[0.0, -0.0, 3.0], [np.nan, 1.0, -2.0], [-0.0, -0.0, 0.0]], np.float64)
    dx = pb.asarray(x, backend=b200)
    assert _same(pb.asnumpy(pb.amin(dx, axis=1)), numpy_backend.reduce(x, (1,), False, None, "min"))
    assert _same(pb.asnumpy(pb.amax(dx, axis=0)), numpy_backend.reduce(x, (0,), False, None, "max"))
    m = np.array([[True, False], [True, True]])
    dm = pb.asarray(m, backend=b200)
    assert _same(pb.asnumpy(pb.amin(dm, axis=1)), m.min(axis=1))
    assert _same(pb.asnumpy(pb.amax(dm, axis=1)), m.max(axis=1))
    count = pb.asnumpy(pb.sum(pb.equal(pb.isfinite(dx), False), dtype=np.float64))
    assert count == 1.0
    y = np.random.default_rng(34).standard_normal((64, 33)).astype(np.float32)
    got = pb.asnumpy(pb.mean(pb.asarray(y, backend=b200), axis=0, keepdims=True))
    assert got.shape == (1, 33)
    assert np.allclose(got, y.mean(axis=0, keepdims=True), rtol=1e-6, atol=1e-7)


def test_gather_views(b200):
    rng = np.random.default_rng(35)
    x = rng.standard_normal((4, 5, 6)).astype(np.float32)
    dx = pb.asarray(x, backend=b200)
    assert _same(pb.asnumpy(pb.transpose(dx)), np.ascontiguousarray(x.transpose()))
    assert _same(pb.asnumpy(pb.transpose(dx, (1, 0, 2))), np.ascontiguousarray(x.transpose(1, 0, 2)))
    m = rng.standard_normal((7, 9))
    dm = pb.asarray(m, backend=b200)
    for k in (-3, 0, 2, 9):
        assert _same(pb.asnumpy(pb.diag(dm, k)), np.diag(m, k).copy())
    # negative strides: reversed rows through the raw gather
    got = b200.gather(dm, (7, 9), 6 * 9, (-9, 1))
    want = numpy_backend.gather(m, (7, 9), 6 * 9, (-9, 1))
    assert _same(pb.asnumpy(pb.wrap(got, (7, 9), m.dtype, b200)), want)


def test_conjugate_gradient_through_the_api(b200):
    """CG on an SPD system, every step on the GPU (matvec, dot, norm and the
    vector updates), against the same iteration in NumPy float64."""
    rng = np.random.default_rng(36)
    n = 512
    q = rng.standard_normal((n, n))
    A = (q @ q.T / n + np.eye(n)).astype(np.float64)
    b = rng.standard_normal(n)

    def cg(xp, A, b, iters):
        x = b * 0.0
        r = b - A @ x
        p = r
        rr = xp.dot(r, r)
        for _ in range(iters):
            Ap = A @ p
            alpha = rr / xp.dot(p, Ap)
            x = x + alpha * p
            r = r - alpha * Ap
            rr_new = xp.dot(r, r)
            p = r + (rr_new / rr) * p
            rr = rr_new
        return x

    dA, db = pb.asarray(A, backend=b200), pb.asarray(b, backend=b200)
    x_gpu = pb.asnumpy(cg(pb, dA, db, 40))
    x_cpu = cg(np, A, b, 40)
    residual = np.linalg.norm(b - A @ x_gpu) / np.linalg.norm(b)
    assert residual < 1e-8
    assert np.allclose(x_gpu, x_cpu, rtol=1e-9, atol=1e-10)
    assert pb.linalg.norm(db - dA @ pb.asarray(x_gpu, backend=b200)).item() / np.linalg.norm(b) < 1e-8


def test_devices_lists_the_b200(b200):
    """pacho_b200.devices(): OpenPacho-style DeviceInfo records of the visible
    B200s (what devices("b200") returns once registered)."""
    import pacho_b200

    listed = pacho_b200.devices("b200")
    assert listed and all(d.vendor == "NVIDIA" and d.fp64 for d in listed)
    assert any("B200" in d.name for d in listed)
