"""Acceptance bounds of the b200 path against the NumPy-backend oracle.

* GEMM/GEMV/DOT, elementwise: |C - C_ref| <= 4 * K * u * (|A| |B|)_ij with
  u = 2^-24 (float32) or 2^-53 (float64); |A||B| is formed in float64.
* Norm, relative: |n - n_ref| <= 8 * u * |n_ref| (NaN matches NaN, Inf Inf).
"""

from __future__ import annotations

import numpy as np

UNIT_ROUNDOFF = {np.dtype(np.float32): 2.0**-24, np.dtype(np.float64): 2.0**-53}


def unit_roundoff(dtype) -> float:
    return UNIT_ROUNDOFF[np.dtype(dtype)]


def gemm_bound(a: np.ndarray, b: np.ndarray, dtype=None) -> np.ndarray:
    """Elementwise 4*K*u*(|A||B|) for ``a @ b`` (broadcasting like matmul)."""
    dtype = np.dtype(dtype or np.result_type(a.dtype, b.dtype))
    k = a.shape[-1]
    absprod = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    return 4.0 * max(k, 1) * unit_roundoff(dtype) * absprod


def gemm_violations(c: np.ndarray, c_ref: np.ndarray, a: np.ndarray, b: np.ndarray) -> int:
    """Number of elements outside the GEMM bound (non-finite must match)."""
    c64, r64 = np.asarray(c, np.float64), np.asarray(c_ref, np.float64)
    bound = gemm_bound(a, b, c_ref.dtype)
    finite = np.isfinite(r64)
    bad = np.zeros(r64.shape, dtype=bool)
    bad |= finite & ~(np.abs(c64 - r64) <= bound)
    bad |= ~finite & ~((np.isnan(r64) & np.isnan(c64)) | (r64 == c64))
    return int(bad.sum())


def norm_violations(n: np.ndarray, n_ref: np.ndarray, dtype=None) -> int:
    """Number of norms outside 8u relative error (non-finite must match)."""
    dtype = np.dtype(dtype or np.asarray(n_ref).dtype)
    n64, r64 = np.asarray(n, np.float64), np.asarray(n_ref, np.float64)
    finite = np.isfinite(r64)
    rel = 8.0 * unit_roundoff(dtype)
    bad = np.zeros(r64.shape, dtype=bool)
    bad |= finite & ~(np.abs(n64 - r64) <= rel * np.abs(r64))
    bad |= ~finite & ~((np.isnan(r64) & np.isnan(n64)) | (r64 == n64))
    return int(bad.sum())
