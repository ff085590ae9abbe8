"""The oracle reproduces the reference's own outputs bit for bit (CPU): the
GEMM and norm hot path, and the elementwise, cast, reduction and gather
operations around it.

The fixtures were produced by the reference itself (OpenPacho on its NumPy
backend) from the reference's hot-path test cases; see golden/make_golden.py.
"""

from __future__ import annotations

import math

import cases
import numpy as np
import pytest

from oracle import exact, numpy_backend, tolerance


def _matmul_inputs():
    for gen in (cases.matmul_cases, cases.empty_cases, cases.batched_cases, cases.gemv_cases,
                cases.dot_cases, cases.signed_cases, cases.special_value_cases):
        yield from gen()
    yield cases.cancellation_case()


def _norm_inputs():
    for gen in (cases.norm_extreme_cases, cases.norm_special_cases, cases.norm_chunk_cases,
                cases.norm_distribution_cases):
        yield from gen()


def test_fixture_covers_every_case(golden):
    data, meta = golden
    names = ([n for n, *_ in _matmul_inputs()] + [n for n, *_ in _norm_inputs()]
             + [c[0] for c in cases.around_cases()])
    assert sorted(names) == sorted(meta) == sorted(data.files)


@pytest.mark.parametrize("case", list(_matmul_inputs()), ids=lambda c: c[0])
def test_oracle_matmul_matches_reference(golden, case):
    data, meta = golden
    name, a, b = case
    assert cases.digest(a, b) == meta[name]["inputs"], "regenerated inputs drifted"
    with np.errstate(all="ignore"):
        got = numpy_backend.matmul(a, b)
    want = data[name]
    assert got.dtype == want.dtype and got.shape == want.shape
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("case", list(_norm_inputs()), ids=lambda c: c[0])
def test_oracle_norm_matches_reference(golden, case):
    data, meta = golden
    name, x, axis, keepdims = case
    assert cases.digest(x) == meta[name]["inputs"]
    got = numpy_backend.norm(x, axis=axis, keepdims=keepdims)
    want = data[name]
    assert got.dtype == want.dtype and got.shape == want.shape
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("case", cases.around_cases(), ids=lambda c: c[0])
def test_oracle_around_path_matches_reference(golden, case):
    """Elementwise, cast, reduction and gather restatements against the
    reference's own outputs: same dtype and shape, equal values with NaN in the
    same places and the same zero signs."""
    data, meta = golden
    name, kind, op, inputs, params = case
    assert cases.digest(*inputs) == meta[name]["inputs"], "regenerated inputs drifted"
    want = data[name]
    if kind == "ew":
        got = numpy_backend.elementwise(op, inputs, want.dtype)
    elif kind == "cast":
        got = numpy_backend.elementwise("cast", inputs, np.dtype(params["dtype"]))
    elif kind == "reduce":
        got = numpy_backend.reduce(inputs[0], params["axis"], False, want.dtype, op)
    else:
        got = numpy_backend.gather(inputs[0], *params["view"])
    assert got.dtype == want.dtype and got.shape == want.shape
    assert np.array_equal(got, want, equal_nan=want.dtype.kind == "f")
    if want.dtype.kind == "f":
        np.testing.assert_array_equal(np.signbit(got), np.signbit(want))


def test_oracle_known_answers():
    # tests/test_stable_norm.py:60-66 of the reference.
    assert numpy_backend.norm(np.asarray([-3.0, 4.0])) == 5.0
    assert numpy_backend.norm(np.asarray([0.0, 0.0])) == 0.0
    assert numpy_backend.norm(np.asarray([np.inf, 1.0])) == np.inf
    assert math.isnan(numpy_backend.norm(np.asarray([np.nan, np.inf])))
    # tests/test_stable_norm.py:36-57: |scale| * sqrt(count) for constant inputs.
    x = np.full((4099,), 1e25, np.float32)
    np.testing.assert_allclose(numpy_backend.norm(x), 1e25 * math.sqrt(4099), rtol=2e-6)


def test_exact_references_agree_with_oracle():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((9, 31)).astype(np.float32)
    b = rng.standard_normal((31, 7)).astype(np.float32)
    c = numpy_backend.matmul(a, b)
    assert tolerance.gemm_violations(c, exact.matmul_exact(a, b).astype(np.float32), a, b) == 0
    x = rng.standard_normal(50) * 1e200
    assert abs(exact.norm_decimal(x) - numpy_backend.norm(x)) <= 8 * 2.0**-53 * exact.norm_decimal(x)
    u, v = rng.standard_normal(40), rng.standard_normal(40)
    assert abs(exact.dot_fraction(u, v) - float(u @ v)) <= 4 * 40 * 2.0**-53 * float(np.abs(u) @ np.abs(v))


def test_tolerance_flags_planted_errors():
    """A mistake planted in the oracle's output is caught by the bounds."""
    rng = np.random.default_rng(6)
    a = rng.standard_normal((8, 64)).astype(np.float32)
    b = rng.standard_normal((64, 8)).astype(np.float32)
    c = numpy_backend.matmul(a, b)
    bad = c.copy()
    bad[3, 4] += 1e-3 * abs(bad[3, 4]) + 1e-3
    assert tolerance.gemm_violations(c, c, a, b) == 0
    assert tolerance.gemm_violations(bad, c, a, b) == 1
    n = numpy_backend.norm(a, axis=1)
    off = n * (1 + 16 * 2.0**-24)
    assert tolerance.norm_violations(n, n) == 0
    assert tolerance.norm_violations(off, n) == n.size
    nan = n.copy()
    nan[0] = np.nan
    assert tolerance.norm_violations(nan, n) == 1
    # With an exact reference, a result closer to exact than a poor reference passes,
    # one further away does not.
    exact_n = n.astype(np.float64)
    poor_ref = (exact_n * (1 + 20 * 2.0**-24)).astype(np.float32)
    assert tolerance.norm_violations(n, poor_ref, exact=exact_n) == 0
    worse = (exact_n * (1 - 40 * 2.0**-24)).astype(np.float32)
    assert tolerance.norm_violations(worse, poor_ref, exact=exact_n) == n.size
