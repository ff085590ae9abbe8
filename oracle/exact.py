"""Exact references for small cases (independent of BLAS).

* ``matmul_exact`` -- every C element as the exactly rounded dot product
  (``math.fsum`` of exact products).  For float32 inputs the products are
  exact in float64, so the result is the correctly rounded sum; this plays the
  role of the reference's exact dyadic oracle
  (benchmarks/gemm_precision_oracle.py:27-93).
* ``dot_fraction`` -- exact rational dot product for float64 inputs (cf.
  benchmarks/fp64_contraction_oracle.py:109-125), rounded once at the end.
* ``norm_decimal`` -- sqrt(sum x^2) in 80-digit Decimal arithmetic
  (cf. benchmarks/accuracy.py:61-66), for norms of extreme magnitudes.
"""

from __future__ import annotations

import math
from decimal import Decimal, localcontext
from fractions import Fraction

import numpy as np


def matmul_exact(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Correctly rounded (to float64) ``a @ b`` for 2-D float32 operands."""
    if a.dtype != np.float32 or b.dtype != np.float32 or a.ndim != 2 or b.ndim != 2:
        raise ValueError("matmul_exact takes 2-D float32 operands")
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    out = np.empty((a.shape[0], b.shape[1]), np.float64)
    for i in range(a.shape[0]):
        prods = a64[i][:, None] * b64  # exact: 24+24 bit significands
        for j in range(b.shape[1]):
            out[i, j] = math.fsum(prods[:, j])
    return out


def dot_fraction(x: np.ndarray, y: np.ndarray) -> float:
    """Exact dot product of float64 vectors, rounded once to float64."""
    total = Fraction(0)
    for u, v in zip(np.asarray(x, np.float64).tolist(), np.asarray(y, np.float64).tolist()):
        total += Fraction(u) * Fraction(v)
    return float(total)


def norm_decimal(x: np.ndarray) -> float:
    """sqrt(sum(x^2)) with 80 significant digits, rounded to float64."""
    with localcontext() as ctx:
        ctx.prec = 80
        total = sum((Decimal(float(v)) ** 2 for v in np.asarray(x).ravel()), Decimal(0))
        return float(total.sqrt())
