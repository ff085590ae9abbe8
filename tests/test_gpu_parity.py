"""CUDA path vs the reference's outputs on the reference's own test cases (B200).

Inputs are regenerated from tests/golden/cases.py (checked against the
fixture's SHA-256); outputs are compared with the golden reference outputs
under the acceptance bounds of oracle/tolerance.py:
GEMM |C - C_ref| <= 4*K*u*(|A||B|), norm relative <= 8u.
"""

from __future__ import annotations

import ctypes as C
import math

import cases
import numpy as np
import pytest

import front as pb
from oracle import exact, numpy_backend, tolerance
from pacho_b200 import _lib

pytestmark = pytest.mark.gpu


def _matmul_cases():
    for gen in (cases.matmul_cases, cases.batched_cases, cases.gemv_cases, cases.dot_cases,
                cases.special_value_cases):
        yield from gen()
    yield cases.cancellation_case()


def _gpu_matmul(backend, a, b):
    return pb.asnumpy(pb.matmul(pb.asarray(a, backend=backend), pb.asarray(b, backend=backend)))


@pytest.mark.parametrize("case", list(_matmul_cases()), ids=lambda c: c[0])
def test_matmul_matches_reference(b200, golden, case):
    data, meta = golden
    name, a, b = case
    assert cases.digest(a, b) == meta[name]["inputs"]
    got = _gpu_matmul(b200, a, b)
    want = data[name]
    assert got.shape == want.shape and got.dtype == want.dtype
    assert tolerance.gemm_violations(got, want, a, b) == 0


@pytest.mark.parametrize("case", list(cases.empty_cases()), ids=lambda c: c[0])
def test_empty_and_k0_products(b200, golden, case):
    data, _ = golden
    name, a, b = case
    got = _gpu_matmul(b200, a, b)
    np.testing.assert_array_equal(got, data[name])
    assert got.dtype == data[name].dtype


@pytest.mark.parametrize("case", list(cases.signed_cases()), ids=lambda c: c[0])
def test_gemv_cancellation_signed_zero_and_nonfinite(b200, golden, case):
    # tests/test_cuda_gemv.py:195-222 of the reference.
    data, _ = golden
    name, a, b = case
    values = _gpu_matmul(b200, a, b)
    np.testing.assert_array_equal(values, data[name])
    assert values[0] == 0 and values[1] == 1
    assert values[2] == 0 and not np.signbit(values[2])
    assert np.isnan(values[3]) and np.isneginf(values[4])


def _norm_cases():
    for gen in (cases.norm_extreme_cases, cases.norm_special_cases, cases.norm_chunk_cases,
                cases.norm_distribution_cases):
        yield from gen()


@pytest.mark.parametrize("case", list(_norm_cases()), ids=lambda c: c[0])
def test_norm_matches_reference(b200, golden, case):
    data, meta = golden
    name, x, axis, keepdims = case
    assert cases.digest(x) == meta[name]["inputs"]
    got = pb.asnumpy(pb.linalg.norm(pb.asarray(x, backend=b200), axis=axis, keepdims=keepdims))
    want = data[name]
    assert got.shape == want.shape and got.dtype == want.dtype
    assert tolerance.norm_violations(got, want) == 0
    # A -0.0 row gives +0.0 (tests/test_cuda.py:462 of the reference).
    assert not np.any(np.signbit(got[got == 0]))


def test_norm_extremes_against_exact_decimal(b200):
    rng = np.random.default_rng(17)
    for dtype, lo, hi in ((np.float32, -35, 35), (np.float64, -300, 300)):
        x = (rng.standard_normal(5000) * 10.0 ** rng.uniform(lo, hi, 5000)).astype(dtype)
        got = pb.linalg.norm(pb.asarray(x, backend=b200)).item()
        ref = exact.norm_decimal(x)
        u = tolerance.unit_roundoff(dtype)
        assert abs(got - ref) <= 2 * u * ref


# ------------------------------------------------- both GEMM kernels --

def _call_gemm_ex(backend, a, b, algo):
    """pb_gemm_ex through the C ABI on uploaded operands."""
    dtype = np.result_type(a.dtype, b.dtype)
    batch = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    m, k = a.shape[-2:]
    n = b.shape[-1]
    from pacho_b200.backend import _matrix_strides

    da, db = backend.upload(a), backend.upload(b)
    out_shape = batch + (m, n)
    dc = backend.empty(out_shape, dtype)
    status = backend._lib.pb_gemm_ex(
        backend._ctx, 0, _lib.dtype_code(dtype), len(batch), _lib.i64_array(batch),
        _lib.i64_array(_matrix_strides(batch, a.shape[:-2])),
        _lib.i64_array(_matrix_strides(batch, b.shape[:-2])), m, n, k,
        C.c_void_p(da.ptr), C.c_void_p(db.ptr), C.c_void_p(dc.ptr), algo)
    _lib.check(status, "pb_gemm_ex")
    return pb.wrap(dc, out_shape, dtype, backend).numpy()


def _gemm_shapes():
    for name, a, b in cases.matmul_cases():
        if a.ndim == 2 and b.ndim == 2:
            yield name, a, b
    for name, a, b in cases.batched_cases():
        if a.ndim >= 2 and b.ndim >= 2 and a.size and b.size:
            yield name, a, b
    yield from cases.special_value_cases()
    rng = np.random.default_rng(11)
    for m, n, k in ((128, 128, 32), (129, 255, 33), (300, 520, 97), (1, 300, 64), (257, 1, 40),
                    (64, 64, 1), (200, 136, 1000), (1, 4099, 3000), (3, 1001, 20000),
                    (8, 64, 5), (5, 2, 70000), (2181, 200, 96), (900, 1100, 500),
                    # two-way K splits: 128- and 64-wide tiles as CTA pairs, and
                    # (N % 4 != 0) through the partial planes and the reduction
                    (1000, 1000, 800), (7680, 48, 384), (1000, 998, 800)):
        yield (f"rand{m}x{n}x{k}", rng.standard_normal((m, k)).astype(np.float32),
               rng.standard_normal((k, n)).astype(np.float32))


@pytest.mark.parametrize("algo", [_lib.PB_GEMM_SIMT, _lib.PB_GEMM_TF32X3, _lib.PB_GEMM_TF32X3_PRESPLIT,
                                  _lib.PB_GEMM_TF32X3_FUSED, _lib.PB_GEMM_DMMA, _lib.PB_GEMM_SKINNY],
                         ids=["simt", "tf32x3", "tf32x3_presplit", "tf32x3_fused", "dmma", "skinny"])
@pytest.mark.parametrize("case", list(_gemm_shapes()), ids=lambda c: c[0])
def test_every_gemm_kernel_on_every_shape(b200, algo, case):
    name, a, b = case
    tf32 = (_lib.PB_GEMM_TF32X3, _lib.PB_GEMM_TF32X3_PRESPLIT, _lib.PB_GEMM_TF32X3_FUSED)
    if algo in tf32 and a.dtype != np.float32:
        pytest.skip("3xTF32 is the float32 kernel")
    if algo == _lib.PB_GEMM_TF32X3_FUSED and a.shape[-1] % 4:
        pytest.skip("the in-kernel A split needs K % 4 == 0")
    if algo == _lib.PB_GEMM_SKINNY and a.shape[-2] > 8:
        pytest.skip("the skinny kernel takes at most 8 rows")
    if algo == _lib.PB_GEMM_DMMA:
        a, b = a.astype(np.float64), b.astype(np.float64)
    got = _call_gemm_ex(b200, a, b, algo)
    with np.errstate(all="ignore"):
        want = numpy_backend.matmul(a, b)
    # Forced 3xTF32 below K=32 carries the split error model (auto sends it to SIMT).
    extra = 16.0 if algo in tf32 and a.shape[-1] < 32 else 0.0
    assert tolerance.gemm_violations(got, want, a, b, extra_u=extra) == 0


@pytest.mark.parametrize("algo", [_lib.PB_GEMM_TF32X3_PRESPLIT, _lib.PB_GEMM_TF32X3_FUSED],
                         ids=["presplit", "fused"])
def test_tf32x3_keeps_float32_accuracy(b200, algo):
    """3xTF32 must be as accurate as float32 GEMM, unlike plain TF32."""
    rng = np.random.default_rng(12)
    a = rng.standard_normal((256, 2048)).astype(np.float32)
    b = rng.standard_normal((2048, 192)).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    got = _call_gemm_ex(b200, a, b, algo).astype(np.float64)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)

    def tf32(x):  # what a single TF32 pass would see (round to 10 mantissa bits)
        bits = x.view(np.uint32).astype(np.uint64)
        return ((bits + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)

    one_pass = tf32(a).astype(np.float64) @ tf32(b).astype(np.float64)
    err_1x = np.linalg.norm(one_pass - ref) / np.linalg.norm(ref)
    sgemm = np.linalg.norm(numpy_backend.matmul(a, b) - ref) / np.linalg.norm(ref)
    assert err_1x > 1e-4  # the check can tell TF32 from float32
    assert err < 1e-6 and err < 4 * sgemm, (err, sgemm, err_1x)


@pytest.mark.parametrize("algo", [_lib.PB_GEMM_TF32X3_PRESPLIT, _lib.PB_GEMM_TF32X3_FUSED],
                         ids=["presplit", "fused"])
def test_tf32x3_error_does_not_grow_with_k(b200, algo):
    """Promotion out of the tensor core's truncating accumulator keeps the
    relative error flat in K (it grew linearly, ~1.9e-5 at K=8192, without)."""
    rng = np.random.default_rng(13)
    errs = []
    for k in (512, 8192):
        a = rng.standard_normal((128, k)).astype(np.float32)
        b = rng.standard_normal((k, 128)).astype(np.float32)
        ref = a.astype(np.float64) @ b.astype(np.float64)
        got = _call_gemm_ex(b200, a, b, algo).astype(np.float64)
        errs.append(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert errs[1] < 1e-6 and errs[1] < 3 * errs[0], errs


@pytest.mark.parametrize("algo", [_lib.PB_GEMM_TF32X3_PRESPLIT, _lib.PB_GEMM_TF32X3_FUSED],
                         ids=["presplit", "fused"])
@pytest.mark.parametrize("shape", [(2048, 2048, 256), (2048, 1024, 256), (2, 600, 300, 1024),
                                   (1024, 1024, 1024)],
                         ids=lambda s: "x".join(map(str, s)))
def test_tf32x3_special_values_match_ieee(b200, algo, shape):
    """Inf/NaN operands give the IEEE classes of the reference's float32 GEMM.

    The 3xTF32 split turns some +-Inf results into NaN (0 * Inf cross terms);
    those tiles are recomputed.  The first two shapes fill every SM without
    splitting K, so the marks come from the tcgen05 epilogues; the batched
    shape splits K four ways and 1024^3 two ways, so they come from the split
    reduction."""
    *batch, m, n, k = shape
    rng = np.random.default_rng(21)
    a = rng.standard_normal((*batch, m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    lead = (0,) * len(batch)
    a[lead + (0, 5)], b[5, 7] = np.inf, 0.0
    b[9, 3], a[lead + (4, 9)] = -np.inf, 0.0
    a[lead + (m - 1, 2)] = np.nan
    a[lead + (300, 20)], a[lead + (300, 21)] = np.inf, -np.inf
    b[20, :] = np.abs(b[20, :]) + 0.5
    b[21, :] = np.abs(b[21, :]) + 0.5
    a[lead + (517, 30)], b[30, :] = np.finfo(np.float32).max, 2.0**-10
    b[40, n - 1] = np.inf
    if batch:
        a[(batch[0] - 1, 77, 11)] = -np.inf
    got = _call_gemm_ex(b200, a, b, algo)
    with np.errstate(all="ignore"):
        want = numpy_backend.matmul(a, b)
    assert np.isnan(want).any() and np.isinf(want).any()
    assert tolerance.gemm_violations(got, want, a, b) == 0
    # The repair leaves its marks at zero: a clean product right after is exact.
    a2 = rng.standard_normal((256, 128)).astype(np.float32)
    b2 = rng.standard_normal((128, 256)).astype(np.float32)
    assert tolerance.gemm_violations(_call_gemm_ex(b200, a2, b2, algo),
                                     numpy_backend.matmul(a2, b2), a2, b2) == 0


@pytest.mark.parametrize("algo", [_lib.PB_GEMM_TF32X3_PRESPLIT, _lib.PB_GEMM_TF32X3_FUSED],
                         ids=["presplit", "fused"])
@pytest.mark.parametrize("shape", [(2048, 2048, 256), (2048, 1024, 256), (2, 600, 300, 1024),
                                   (1024, 1024, 1024)],
                         ids=lambda s: "x".join(map(str, s)))
def test_tf32x3_tiny_operands_keep_float32_accuracy(b200, algo, shape):
    """Operands below 2^-57 (products that would be subnormal on the tensor
    core, subnormal inputs) still meet the float32 GEMM bound."""
    *batch, m, n, k = shape
    rng = np.random.default_rng(22)
    a = rng.standard_normal((*batch, m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    lead = (0,) * len(batch)
    a[lead + (5,)] *= np.float32(2.0**-70)         # tiny row ...
    b[:, 9] *= np.float32(2.0**-70)                # ... times tiny column: subnormal products
    a[lead + (m - 3,)] = (rng.standard_normal(k) * 2.0**-135).astype(np.float32)  # subnormals
    b[17, n - 2] = np.float32(2.0**-140)
    a[lead + (200, 17)] = np.float32(3.0)
    got = _call_gemm_ex(b200, a, b, algo)
    want = numpy_backend.matmul(a, b)
    assert want[lead + (5, 9)] != 0 and abs(want[lead + (5, 9)]) < 2.0**-126
    assert tolerance.gemm_violations(got, want, a, b) == 0


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("shapes", [((16384,), (16384, 4096)), ((3000,), (5, 3000, 777)),
                                    ((4, 513), (513, 9000)), ((2, 7, 2000), (2000, 130)),
                                    ((1, 65536), (3, 65536, 12))],
                         ids=lambda s: "@".join("x".join(map(str, t)) for t in s))
def test_vector_and_few_row_products(b200, dtype, shapes):
    """Vector @ matrix and products with at most 8 rows (the skinny kernel),
    broadcast batches, unaligned N and K split over blocks, via pb.matmul."""
    rng = np.random.default_rng(23)
    a = rng.standard_normal(shapes[0]).astype(dtype)
    b = rng.standard_normal(shapes[1]).astype(dtype)
    a.flat[7] = np.inf
    got = _gpu_matmul(b200, a, b)
    with np.errstate(all="ignore"):
        want = numpy_backend.matmul(a, b)
    assert got.shape == want.shape
    assert tolerance.gemm_violations(got, want, a, b) == 0


def test_products_overwrite_nan_and_inf_destinations(b200, monkeypatch):
    # tests/test_cuda.py:345-389 of the reference: every output is written.
    for dtype in (np.float32, np.float64):
        for poison in (np.nan, np.inf):
            for name, a, b in list(cases.matmul_cases())[:4] + [("big", np.ones((130, 70), dtype),
                                                                  np.ones((70, 260), dtype))]:
                a, b = a.astype(dtype), b.astype(dtype)
                expected = numpy_backend.matmul(a, b)
                dest = b200.full(expected.shape, poison, dtype)
                original = b200.empty

                def poisoned(shape, requested, dest=dest, shape0=expected.shape):
                    if tuple(shape) == shape0 and np.dtype(requested) == np.dtype(dtype):
                        return dest
                    return original(shape, requested)

                with monkeypatch.context() as patch:
                    patch.setattr(b200, "empty", poisoned)
                    got = _gpu_matmul(b200, a, b)
                assert np.isfinite(got).all(), name
                assert tolerance.gemm_violations(got, expected, a, b) == 0


def test_norm_strided_general_axes(b200):
    rng = np.random.default_rng(21)
    x = rng.standard_normal((3, 5, 7, 2))
    with pytest.raises(ValueError):  # linalg.py:11 of the reference: 1 or 2 axes only
        pb.linalg.norm(pb.asarray(x, backend=b200), axis=(0, 1, 3))
    for axis in ((0, 2), (1, 3), (0, 3), 1, -1):
        for keep in (False, True):
            got = pb.asnumpy(pb.linalg.norm(pb.asarray(x, backend=b200), axis=axis, keepdims=keep))
            want = numpy_backend.norm(x, axis=axis, keepdims=keep)
            assert got.shape == want.shape
            assert tolerance.norm_violations(got, want) == 0


def test_norm_columns_split_over_blocks(b200):
    # Reduced axis first with few outputs: split across blocks + merge.
    rng = np.random.default_rng(22)
    for dtype in (np.float32, np.float64):
        x = (rng.standard_normal((20000, 3)) * 10.0 ** rng.uniform(-20, 20, (20000, 3))).astype(dtype)
        x[5, 1] = np.inf
        x[7, 2] = np.nan
        got = pb.asnumpy(pb.linalg.norm(pb.asarray(x, backend=b200), axis=0))
        want = numpy_backend.norm(x, axis=0)
        # The float32 reference is itself ~6e-7 off here; the exact norm attributes it.
        ex = np.array([exact.norm_decimal(x[:, j]) for j in range(3)])
        assert tolerance.norm_violations(got, want, exact=ex) == 0
        assert np.isinf(got[1]) and np.isnan(got[2])


def test_repeated_calls_are_deterministic(b200):
    rng = np.random.default_rng(23)
    x = rng.standard_normal(1 << 22).astype(np.float32)
    y = rng.standard_normal(1 << 22).astype(np.float32)
    dx, dy = pb.asarray(x, backend=b200), pb.asarray(y, backend=b200)
    dots = {pb.matmul(dx, dy).item() for _ in range(5)}
    norms = {pb.linalg.norm(dx).item() for _ in range(5)}
    assert len(dots) == 1 and len(norms) == 1
    assert math.isclose(next(iter(norms)), float(np.linalg.norm(x.astype(np.float64))), rel_tol=1e-7)
