"""Restatement of OpenPacho's NumPy backend (test oracle): matmul and norm on
the path, and the elementwise, gather and reduce operations around it.

Each function cites the reference lines it follows.  Inputs and outputs are
NumPy arrays; shapes and dtypes follow the reference's front end
(src/openpacho/_array.py:241-281, 389-479, src/openpacho/linalg.py:8-35).
Test infrastructure only: nothing in the product imports this module.
"""

from __future__ import annotations

from math import prod

import numpy as np


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``a @ b`` in the promoted dtype.

    src/openpacho/_array.py:469 promotes with ``np.result_type``;
    src/openpacho/backends.py:139-142 computes ``a @ b`` and casts to dtype.
    """
    dtype = np.result_type(a.dtype, b.dtype)
    a, b = a.astype(dtype, copy=False), b.astype(dtype, copy=False)
    return np.asarray(a @ b, dtype=dtype)


def dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """src/openpacho/_array.py:482-491: for 1-D/2-D operands ``dot`` is matmul."""
    if a.ndim > 2 or b.ndim > 2:
        raise NotImplementedError("Higher-rank dot differs from batched matmul")
    return matmul(a, b)


def _axes(axis, ndim):
    """src/openpacho/_array.py:376-386."""
    if axis is None:
        return tuple(range(ndim))
    values = axis if isinstance(axis, tuple) else (axis,)
    if ndim == 0 and not isinstance(axis, tuple) and axis in (0, -1):
        return ()
    values = tuple(int(i) % ndim for i in values)
    if len(set(values)) != len(values):
        raise ValueError("duplicate reduction axis")
    return tuple(sorted(values))


def norm_data(data: np.ndarray, axes: tuple, dtype) -> np.ndarray:
    """NumPy branch of norm_data, returning the flat (count,) result.

    src/openpacho/_norm.py:41-43: empty output or empty reduction -> zeros.
    src/openpacho/_norm.py:44-52: scale = max|x| over axes; x/scale where
    scale != 0 else 0; sum of squares in ``dtype``; scale*sqrt(total); where
    the scale is infinite the result is the scale.
    """
    dtype = np.dtype(dtype)
    shape = data.shape
    count = prod(d for i, d in enumerate(shape) if i not in axes)
    reduced = prod(shape[i] for i in axes)
    if not count or not reduced:
        return np.zeros((count,), dtype=dtype)
    scale = np.max(np.abs(data), axis=axes, keepdims=True)
    with np.errstate(all="ignore"):
        normalized = np.divide(data, scale, out=np.zeros_like(data), where=scale != 0)
        total = np.sum(normalized * normalized, axis=axes, keepdims=True, dtype=dtype)
        result = scale * np.sqrt(total)
    result = np.where(np.isinf(scale), scale, result)
    return np.asarray(result, dtype=dtype).reshape(-1)


def norm(x: np.ndarray, axis=None, keepdims=False) -> np.ndarray:
    """``linalg.norm(x, axis=axis, keepdims=keepdims)`` on the NumPy backend
    (src/openpacho/linalg.py:8-35 with ord=None)."""
    x = np.asarray(x)
    if x.dtype.kind != "f":
        x = x.astype(np.float64)
    axes = _axes(axis, x.ndim)
    shape = (
        tuple(1 if i in axes else d for i, d in enumerate(x.shape))
        if keepdims
        else tuple(d for i, d in enumerate(x.shape) if i not in axes)
    )
    return norm_data(x, axes, x.dtype).reshape(shape)


def elementwise(name: str, args, dtype) -> np.ndarray:
    """src/openpacho/backends.py:109-116: ``cast`` is astype, ``where`` is
    np.where, everything else the NumPy ufunc of that name, with floating
    point warnings silenced, then converted to the result dtype."""
    values = [np.asarray(a) for a in args]
    if name == "cast":
        value = values[0].astype(dtype)
    else:
        with np.errstate(all="ignore"):
            value = getattr(np, name)(*values)
    return np.asarray(value, dtype=dtype)


def gather(a: np.ndarray, shape, offset: int, strides) -> np.ndarray:
    """src/openpacho/backends.py:118-128: a strided view of the flat storage,
    copied."""
    flat = np.ascontiguousarray(a).reshape(-1)
    if not prod(shape):
        return np.empty(tuple(shape), dtype=a.dtype)
    view = np.lib.stride_tricks.as_strided(flat[offset:], shape=tuple(shape),
                                           strides=tuple(s * a.dtype.itemsize for s in strides),
                                           writeable=False)
    return np.array(view, copy=True)


def _extreme(value: np.ndarray, axes, keepdims, operation) -> np.ndarray:
    """src/openpacho/_reductions.py:75-90: NumPy extrema, with zero ties
    resolved to -0 for min and +0 for max."""
    function = np.min if operation == "min" else np.max
    result = function(value, axis=axes, keepdims=keepdims)
    if value.dtype.kind == "f" and np.any(result == 0):
        negative = np.signbit(value)
        if operation == "min":
            sign = np.any((value == 0) & negative, axis=axes, keepdims=keepdims)
        else:
            sign = ~np.any((value == 0) & ~negative, axis=axes, keepdims=keepdims)
        zero = np.copysign(np.zeros_like(result), np.where(sign, -1, 1))
        result = np.where(result == 0, zero, result).astype(value.dtype, copy=False)
    return np.asarray(result, dtype=value.dtype)


def reduce(a: np.ndarray, axes, keepdims, dtype, operation="sum") -> np.ndarray:
    """src/openpacho/backends.py:130-136: np.sum with the requested dtype, or
    the extrema above."""
    axes = tuple(axes)
    if operation != "sum":
        return _extreme(a, axes, keepdims, operation)
    return np.asarray(np.sum(a, axis=axes, keepdims=keepdims, dtype=dtype))
