"""Acceptance bounds of the b200 path against the NumPy-backend oracle.

* GEMM/GEMV/DOT, elementwise: |C - C_ref| <= 4 * K * u * (|A| |B|)_ij with
  u = 2^-24 (float32) or 2^-53 (float64); |A||B| is formed in float64.  Plus
  the underflow term of the same error analysis, K * eta with eta the
  smallest subnormal: a product in the subnormal range is rounded to
  multiples of eta (an error of up to eta/2 that no relative bound covers),
  so two correct implementations can differ by K * eta there.  For outputs
  in the normal range the term is below 1e-41 (float32).
* Norm, relative: |n - n_ref| <= 8 * u * |n_ref| (NaN matches NaN, Inf Inf).
  Where the NumPy reference is itself further than that from the exact value
  (float32 normalisation and squaring, src/openpacho/_norm.py:47-49), an
  optional exact reference makes the error attributable: a result that is no
  further from the exact norm than the reference is (or within 2u of it)
  also passes.
* Forced 3xTF32 at tiny K: each product carries up to ~12u of split error
  (dropped lo*lo, tf32 rounding of the lo parts), so ``extra_u=16`` widens the
  bound by 16*u*(|A||B|); automatic dispatch sends K < 32 to the SIMT kernel.
"""

from __future__ import annotations

import numpy as np

UNIT_ROUNDOFF = {np.dtype(np.float32): 2.0**-24, np.dtype(np.float64): 2.0**-53}


def unit_roundoff(dtype) -> float:
    return UNIT_ROUNDOFF[np.dtype(dtype)]


def gemm_bound(a: np.ndarray, b: np.ndarray, dtype=None, extra_u: float = 0.0) -> np.ndarray:
    """Elementwise (4*K + extra_u)*u*(|A||B|) + K*eta for ``a @ b`` (broadcasting like matmul)."""
    dtype = np.dtype(dtype or np.result_type(a.dtype, b.dtype))
    k = a.shape[-1]
    absprod = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    eta = float(np.finfo(dtype).smallest_subnormal)
    return (4.0 * max(k, 1) + extra_u) * unit_roundoff(dtype) * absprod + max(k, 1) * eta


def gemm_violations(c: np.ndarray, c_ref: np.ndarray, a: np.ndarray, b: np.ndarray,
                    extra_u: float = 0.0) -> int:
    """Number of elements outside the GEMM bound (non-finite must match)."""
    c64, r64 = np.asarray(c, np.float64), np.asarray(c_ref, np.float64)
    bound = gemm_bound(a, b, c_ref.dtype, extra_u)
    finite = np.isfinite(r64)
    bad = np.zeros(r64.shape, dtype=bool)
    bad |= finite & ~(np.abs(c64 - r64) <= bound)
    bad |= ~finite & ~((np.isnan(r64) & np.isnan(c64)) | (r64 == c64))
    return int(bad.sum())


def norm_violations(n: np.ndarray, n_ref: np.ndarray, dtype=None, exact=None) -> int:
    """Number of norms outside 8u relative error (non-finite must match).

    ``exact`` (float64, same shape) lets a result pass that is at least as
    close to the exact norm as the reference (or within 2u of it), where the
    reference itself is off by more than 8u."""
    dtype = np.dtype(dtype or np.asarray(n_ref).dtype)
    n64, r64 = np.asarray(n, np.float64), np.asarray(n_ref, np.float64)
    finite = np.isfinite(r64)
    u = unit_roundoff(dtype)
    ok = np.abs(n64 - r64) <= 8.0 * u * np.abs(r64)
    if exact is not None:
        e64 = np.asarray(exact, np.float64)
        allowed = np.maximum(np.abs(r64 - e64), 2.0 * u * np.abs(e64))
        ok |= np.abs(n64 - e64) <= allowed
    bad = np.zeros(r64.shape, dtype=bool)
    bad |= finite & ~ok
    bad |= ~finite & ~((np.isnan(r64) & np.isnan(n64)) | (r64 == n64))
    return int(bad.sum())
