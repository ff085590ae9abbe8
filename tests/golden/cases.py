"""Deterministic inputs of the reference's own hot-path test cases.

Shared by ``make_golden.py`` (which runs the reference on them once, in the
build container) and the tests (which regenerate them, check their SHA-256
against the fixture and compare outputs).  Each generator cites the reference
test it reproduces.
"""

from __future__ import annotations

import hashlib

import numpy as np

DTYPES = (np.float32, np.float64)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


# tests/test_cuda.py:280-318 (_MATMUL_CASES), float32 and float64.
def matmul_cases():
    base = (
        ("vector", np.asarray([1.25, -2.0, 0.5, 3.0, -1.0, 2.5, 4.0]),
         np.asarray([-2.0, 3.0, 1.5, -0.5, 2.0, 0.25, -1.0])),
        ("gemv", np.arange(3 * 5, dtype=np.float64).reshape(3, 5) / 11,
         np.asarray([1.0, -2.0, 0.5, 3.0, -1.5])),
        ("vecmat", np.asarray([1.0, -2.0, 0.5, 3.0, -1.5]),
         np.arange(5 * 4, dtype=np.float64).reshape(5, 4) / 13),
        ("irregular_gemm", np.arange(5 * 7, dtype=np.float64).reshape(5, 7) / 17,
         np.arange(7 * 3, dtype=np.float64).reshape(7, 3) / 19),
        ("odd_tile_gemm", np.arange(33 * 17, dtype=np.float64).reshape(33, 17) / 101,
         np.arange(17 * 65, dtype=np.float64).reshape(17, 65) / 103),
        ("large_odd_gemm", np.arange(65 * 63, dtype=np.float64).reshape(65, 63) / 107,
         np.arange(63 * 97, dtype=np.float64).reshape(63, 97) / 109),
    )
    for dtype in DTYPES:
        for name, a, b in base:
            yield f"{name}_{np.dtype(dtype).name}", a.astype(dtype), b.astype(dtype)


# tests/test_cuda.py:326-342 (empty and K=0 products).
def empty_cases():
    shapes = (
        ("zero_rows", (0, 5), (5, 3)),
        ("zero_inner", (2, 0), (0, 3)),
        ("row_k0", (1, 0), (0, 7)),
        ("zero_columns", (4, 3), (3, 0)),
        ("empty_vector", (0,), (0,)),
        ("empty_gemv", (2, 0), (0,)),
    )
    for dtype in DTYPES:
        for name, sa, sb in shapes:
            yield f"{name}_{np.dtype(dtype).name}", np.zeros(sa, dtype), np.zeros(sb, dtype)


# tests/test_cuda.py:392-406 (batched broadcast products), rng 830.
BATCHED_SHAPES = (
    ((3, 33, 17), (3, 17, 65)),
    ((2, 1, 33, 17), (1, 3, 17, 65)),
    ((2, 5, 7), (7, 3)),
    ((5, 7), (2, 7, 3)),
    ((2, 5, 7), (7,)),
    ((7,), (2, 7, 3)),
    ((2, 5, 0), (2, 0, 3)),
    ((0, 5, 7), (1, 7, 3)),
)


def batched_cases():
    for dtype in DTYPES:
        for i, shapes in enumerate(BATCHED_SHAPES):
            rng = np.random.default_rng(830)
            left, right = (rng.normal(size=s).astype(dtype) for s in shapes)
            yield f"batched{i}_{np.dtype(dtype).name}", left, right


# tests/test_cuda_gemv.py:133-159 (irregular GEMV rows, batches, boundaries).
GEMV_SHAPES = ((33, 17), (129, 67), (33, 255), (33, 256), (33, 257), (513, 1023), (3, 4099),
               (2, 3, 257), (2, 1, 513))


def gemv_cases():
    for dtype in DTYPES:
        for shape in GEMV_SHAPES:
            rng = np.random.default_rng(9101 + len(shape) + shape[-1])
            left = rng.uniform(-1, 1, shape).astype(dtype)
            right = rng.uniform(-1, 1, shape[-1]).astype(dtype)
            yield f"gemv{'x'.join(map(str, shape))}_{np.dtype(dtype).name}", left, right


# tests/test_cuda_gemv.py:174-192 (DOT tails, boundaries, long partials).
DOT_LENGTHS = (63, 64, 65, 4096, 4097, 9001)


def dot_cases():
    for dtype in DTYPES:
        for length in DOT_LENGTHS:
            rng = np.random.default_rng(9102 + length)
            left = rng.uniform(-1, 1, length).astype(dtype)
            right = rng.uniform(-1, 1, length).astype(dtype)
            yield f"dot{length}_{np.dtype(dtype).name}", left, right


# tests/test_cuda_gemv.py:162-171 (seed-941 cancellation regression).
def cancellation_case():
    rng = np.random.default_rng(941)
    left = rng.uniform(-0.5, 0.5, (129, 8193)).astype(np.float32)
    right = rng.uniform(-0.5, 0.5, 8193).astype(np.float32)
    return "cancel941_float32", left, right


# tests/test_rectangular_gemm.py:88-101 (Inf, NaN and the smallest subnormal
# against [0, 1, -1] through a skinny GEMM), then the same kinds of special
# values at tensor-core shapes: Inf * 0, Inf - Inf, a NaN row, a signed-Inf
# column, a broadcast batch, and an operand at the largest finite magnitude.
def special_value_cases():
    for dtype in DTYPES:
        left = np.zeros((33, 4081), dtype=dtype)
        right = np.zeros((4081, 257), dtype=dtype)
        left[0, 0], left[1, 0] = np.inf, np.nan
        left[2, 0] = np.nextafter(dtype(0), dtype(1))
        right[0, :3] = [0, 1, -1]
        yield f"special_rect_{np.dtype(dtype).name}", left, right
    for dtype in DTYPES:
        rng = np.random.default_rng(12)
        a = rng.standard_normal((260, 96)).astype(dtype)
        b = rng.standard_normal((96, 140)).astype(dtype)
        a[0, 5], b[5, 7] = np.inf, 0.0           # row 0 +-Inf; (0, 7) is Inf * 0
        b[9, 3], a[4, 9] = -np.inf, 0.0          # column 3 +-Inf; (4, 3) is 0 * -Inf
        a[11, 2] = np.nan                        # row 11 NaN
        a[13, 20], a[13, 21] = np.inf, -np.inf   # row 13 Inf - Inf where both b > 0
        b[20, :] = np.abs(b[20, :]) + 0.5
        b[21, :] = np.abs(b[21, :]) + 0.5
        a[17, 30], b[30, :] = np.finfo(dtype).max, 2.0**-10  # finite products near the top
        yield f"special_tc_{np.dtype(dtype).name}", a, b
        a = rng.standard_normal((3, 130, 64)).astype(dtype)
        b = rng.standard_normal((64, 136)).astype(dtype)
        a[1, 7, 3], a[2, 129, 0] = np.inf, np.nan
        b[10, 135] = -np.inf
        yield f"special_batched_{np.dtype(dtype).name}", a, b


# tests/test_cuda_gemv.py:195-222 (exact cancellation, signed zero, Inf/NaN rows).
def signed_cases():
    for dtype in DTYPES:
        left = np.zeros((5, 257), dtype=dtype)
        right = np.zeros(257, dtype=dtype)
        left[0, :4] = np.asarray([4096, -4096, 3, -3], dtype=dtype)
        right[:4] = np.asarray([1, 1, 1, 1], dtype=dtype)
        left[1, 20], right[20] = np.asarray(2.0**60, dtype=dtype), np.asarray(2.0**-60, dtype=dtype)
        left[2, 10], right[10] = np.asarray(-0.0, dtype=dtype), np.asarray(1.0, dtype=dtype)
        left[2, 11], right[11] = np.asarray(0.0, dtype=dtype), np.asarray(1.0, dtype=dtype)
        left[3, 60], right[60] = np.asarray(np.inf, dtype=dtype), np.asarray(0.0, dtype=dtype)
        left[4, 61], right[61] = np.asarray(-np.inf, dtype=dtype), np.asarray(1.0, dtype=dtype)
        yield f"signed_{np.dtype(dtype).name}", left, right


# tests/test_stable_norm.py:30-57 (extreme constant inputs; output via keepdims).
NORM_EXTREME_SHAPES = (((2,), None), ((3, 5, 7), (2, 0)), ((4099,), None), ((2, 0, 5), 1),
                       ((), None))


def norm_extreme_cases():
    for dtype, small, large in ((np.float32, 1e-25, 1e25), (np.float64, 1e-200, 1e200)):
        for shape, axis in NORM_EXTREME_SHAPES:
            for tag, scale in (("small", small), ("large", large), ("zero", 0.0)):
                name = f"ext_{np.dtype(dtype).name}_{'x'.join(map(str, shape)) or 'scalar'}_{tag}"
                yield name, np.full(shape, scale, dtype=dtype), axis, True


# tests/test_stable_norm.py:60-66 (specials; float64 as np.asarray gives).
def norm_special_cases():
    values = (("zeros", [0.0, 0.0]), ("inf", [np.inf, 1.0]), ("naninf", [np.nan, np.inf]),
              ("345", [-3.0, 4.0]))
    for name, v in values:
        yield f"special_{name}", np.asarray(v), None, False


# tests/test_cuda.py:442-465 (chunk boundaries, NaN/Inf precedence, -0.0 rows).
def norm_chunk_cases():
    for dtype in DTYPES:
        small, large = (1e-25, 1e25) if dtype == np.float32 else (1e-200, 1e200)
        for length in (4096, 4097, 8193):
            host = np.zeros((6, length), dtype=dtype)
            host[0, [0, -1]] = large
            host[1, [0, -1]] = small
            host[2, -1] = np.inf
            host[3, 0], host[3, -1] = np.nan, np.inf
            host[4, 0], host[4, -1] = np.inf, np.nan
            host[5, [0, -1]] = -0.0
            yield f"chunk{length}_{np.dtype(dtype).name}", host, 1, True


# BASELINE config 4 distribution at a test-sized scale: N(0,1) * 10^U(lo,hi).
def norm_distribution_cases():
    for dtype, lo, hi in ((np.float32, -35, 35), (np.float64, -300, 300)):
        rng = np.random.default_rng(3)
        n = 1 << 16
        x = (rng.standard_normal(n) * 10.0 ** rng.uniform(lo, hi, n)).astype(dtype)
        yield f"dist_full_{np.dtype(dtype).name}", x, None, False
        rows = x.reshape(64, 1024)
        yield f"dist_rows_{np.dtype(dtype).name}", rows, 1, False
        yield f"dist_cols_{np.dtype(dtype).name}", rows, 0, False


# ------------------------------------------------ around the path --------
#
# Elementwise operations, casts, reductions and strided gathers (the rows
# widened beyond the GEMM/norm path).  Each case is (name, kind, op, inputs,
# params): kind "ew" calls the public ufunc `op` on the inputs, "cast" is
# astype(params["dtype"]), "reduce" is sum/min/max over params["axis"],
# "gather" is transpose(params["axes"]) or diag(k=params["k"]) together with
# the (shape, offset, strides) view the backend is asked to copy.
def around_cases():
    out = []
    for dtype in DTYPES:
        tag = np.dtype(dtype).name
        # tests/test_extrema.py:61-80: zero ties, NaN and infinities across chunks.
        host = np.zeros((5, 8193), dtype=dtype)
        host[0, :4096] = -0.0
        host[1] = -0.0
        host[3, 4097] = np.nan
        host[4, 0], host[4, -1] = -np.inf, np.inf
        out.append((f"extrema_min_{tag}", "reduce", "min", [host], {"axis": (1,)}))
        out.append((f"extrema_max_{tag}", "reduce", "max", [host], {"axis": (1,)}))
        # tests/test_where.py:43-56: numeric truth, selected non-finites, zero sign.
        cond = np.array([0, -0.0, 0.5, np.nan, np.inf, -np.inf], dtype=dtype)
        left = np.array([np.nan, np.nan, np.nan, -0.0, np.inf, -np.inf], dtype=dtype)
        right = np.array([0, -0.0, 42, 13, np.nan, np.nan], dtype=dtype)
        out.append((f"where_{tag}", "ew", "where", [cond, left, right], {}))
        # Arithmetic, comparisons and transcendentals over special values.
        rng = np.random.default_rng(31)
        x = rng.standard_normal((4, 1, 37)).astype(dtype)
        y = rng.standard_normal((3, 37)).astype(dtype)
        x.reshape(-1)[:6] = [np.inf, -np.inf, np.nan, -0.0, 0.0, np.finfo(dtype).tiny / 8]
        y.reshape(-1)[:6] = [0.0, -0.0, 2.0, np.inf, -3.5, 1e-30]
        for op in ("add", "subtract", "multiply", "true_divide", "power", "equal", "less",
                   "greater_equal"):
            out.append((f"ew_{op}_{tag}", "ew", op, [x, y], {}))
        for op in ("exp", "log", "sqrt", "sin", "tanh", "absolute", "negative", "isfinite"):
            out.append((f"ew_{op}_{tag}", "ew", op, [x], {}))
        # Sums over axis sets, all axes included.
        z = rng.standard_normal((7, 9, 11)).astype(dtype)
        out.append((f"sum_axes02_{tag}", "reduce", "sum", [z], {"axis": (0, 2)}))
        out.append((f"sum_all_{tag}", "reduce", "sum", [z], {"axis": (0, 1, 2)}))
        # Strided gathers: a transpose and two diagonals.
        g = rng.standard_normal((3, 4, 5)).astype(dtype)
        out.append((f"transpose_{tag}", "gather", "transpose", [g],
                    {"axes": (2, 0, 1), "view": ((5, 3, 4), 0, (1, 20, 5))}))
        d = rng.standard_normal((4, 6)).astype(dtype)
        out.append((f"diag0_{tag}", "gather", "diag", [d], {"k": 0, "view": ((4,), 0, (7,))}))
        out.append((f"diag1_{tag}", "gather", "diag", [d], {"k": 1, "view": ((4,), 1, (7,))}))
    # tests/test_edge_cases.py:81-83: astype(bool) of NaN and signed values;
    # tests/test_edge_cases.py:124-131: broadcasting across ranks and a 0-d operand.
    values = np.asarray([0.0, 2.0, -1.0, np.nan], dtype=np.float32)
    out.append(("cast_bool_float32", "cast", "cast", [values], {"dtype": "bool"}))
    wide = np.asarray([1e39, -1e39, 3.0, 1e-46, np.nan], dtype=np.float64)
    out.append(("cast_float32_float64", "cast", "cast", [wide], {"dtype": "float32"}))
    lh = np.arange(6, dtype=np.float32).reshape(2, 1, 3)
    rh = np.arange(12, dtype=np.float32).reshape(4, 3)
    out.append(("broadcast_add_float32", "ew", "add", [lh, rh], {}))
    out.append(("scalar_multiply_float32", "ew", "multiply", [lh, np.asarray(2.0, np.float32)], {}))
    return out
