"""OpenPacho's public array API for the linear-algebra path, over b200.

A self-contained mirror of the parts of OpenPacho's front end that reach the
hot path, with the same names, argument meaning and errors:

* ``ndarray`` -- C-contiguous array owned by one backend
  (src/openpacho/_array.py:31-199), with ``@`` through ``__array_ufunc__``
  (:104-114) and ``np.dot``/``np.linalg.norm`` through ``__array_function__``;
* ``array``/``asarray``/``asnumpy``/``to_backend``/``empty``/``full``/
  ``zeros``/``ones`` (:205-319), ``reshape`` (:337-352);
* ``matmul(a, b, *, padding=False)`` and ``dot`` (:457-491);
* the elementwise ufuncs of src/openpacho/_ops.py:5-29 (``+ - * / **``,
  comparisons, ``sqrt``/``exp``/... and ``where``, :241-281), ``astype``,
  ``sum``/``mean``/``amin``/``amax`` (:389-454), ``transpose``/``diag``
  (:355-366, 494-503), ``zeros_like``/``ones_like`` (:312-319);
* backend selection ``get_backend``/``set_backend``/``use_backend``/
  ``synchronize`` (src/openpacho/backends.py:153-235) for ``"b200"``.

Use it where OpenPacho itself is not installed; where it is, call
:func:`pacho_b200.register` and use OpenPacho directly.  Only b200 backends
exist here: there is no host (NumPy) compute backend in this package.
"""

from __future__ import annotations

import operator
from contextlib import contextmanager
from contextvars import ContextVar
from functools import lru_cache
from math import prod

import numpy as np
from numpy.lib.mixins import NDArrayOperatorsMixin

from .backend import B200Backend
from . import exceptions as _exc

_FUNCTIONS = {}

# src/openpacho/_ops.py:5-29
UFUNCS = {
    name: getattr(np, name)
    for name in (
        "add", "subtract", "multiply", "true_divide", "power", "negative", "positive",
        "absolute", "sqrt", "exp", "log", "sin", "cos", "tanh", "equal", "not_equal", "less",
        "less_equal", "greater", "greater_equal", "isfinite",
    )
}


# ------------------------------------------------------------ backends --

@lru_cache(maxsize=8)
def _get_b200(device):
    return B200Backend(device)


_DEFAULT: ContextVar = ContextVar("pacho_b200_backend", default=None)


def get_backend(backend=None, *, device=None):
    """Resolve ``"b200"``/a backend object/an array to its backend
    (backends.get_backend, src/openpacho/backends.py:178-214)."""
    if isinstance(backend, ndarray):
        if device is not None:
            raise ValueError("An array's backend cannot be reconfigured")
        return backend._backend
    if isinstance(backend, B200Backend):
        if device is not None:
            raise ValueError("device cannot accompany an existing backend")
        return backend
    if backend is None:
        if device is not None:
            raise ValueError("device requires backend='b200'")
        selected = _DEFAULT.get()
        return selected if selected is not None else _get_b200(None)
    if backend == "b200":
        return _get_b200(None if device is None else str(device))
    raise ValueError("backend must be 'b200' or a B200Backend object")


def set_backend(backend, *, device=None):
    selected = get_backend(backend, device=device)
    _DEFAULT.set(selected)
    return selected


@contextmanager
def use_backend(backend, *, device=None):
    selected = get_backend(backend, device=device)
    token = _DEFAULT.set(selected)
    try:
        yield selected
    finally:
        _DEFAULT.reset(token)


def synchronize(backend=None):
    get_backend(backend).synchronize()


# --------------------------------------------------------------- array --

def _shape(value):
    if isinstance(value, (int, np.integer)):
        value = (value,)
    result = tuple(operator.index(d) for d in value)
    if any(d < 0 for d in result):
        raise ValueError("negative dimensions are not allowed")
    return result


class ndarray(NDArrayOperatorsMixin):
    """C-contiguous array owned by one backend. Construct with array()/asarray()."""

    __array_priority__ = 1000

    def __init__(self, *args, **kwargs):
        raise TypeError("Use pacho_b200.array(), asarray(), zeros(), or ones()")

    @classmethod
    def _wrap(cls, data, shape, dtype, backend):
        obj = object.__new__(cls)
        obj._data, obj._shape, obj._dtype, obj._backend = data, tuple(shape), np.dtype(dtype), backend
        return obj

    shape = property(lambda self: self._shape)
    dtype = property(lambda self: self._dtype)
    ndim = property(lambda self: len(self._shape))
    size = property(lambda self: prod(self._shape))
    nbytes = property(lambda self: self.size * self._dtype.itemsize)
    backend = property(lambda self: self._backend.name)
    device = property(lambda self: self._backend.device)

    def __repr__(self):
        return (f"pacho_b200.ndarray(shape={self.shape}, dtype={self.dtype}, "
                f"backend={self.backend!r}, device={self.device!r})")

    def __len__(self):
        if not self.ndim:
            raise TypeError("len() of unsized object")
        return self.shape[0]

    def __bool__(self):
        raise ValueError("Array truth is ambiguous; transfer a scalar explicitly with .item()")

    def __array__(self, dtype=None, copy=None):
        raise TypeError("Implicit host conversion is disabled. Use asnumpy(a) or a.to_host()")

    def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
        if method != "__call__" or kwargs.get("out") is not None:
            return NotImplemented
        kwargs.pop("out", None)
        if ufunc is np.matmul:
            return matmul(*inputs, **kwargs)
        if ufunc not in UFUNCS.values():
            return NotImplemented
        if kwargs:
            raise NotImplementedError(f"ufunc options {tuple(kwargs)} are not supported")
        return _elementwise(ufunc, *inputs)

    def __array_function__(self, func, types, args, kwargs):
        if func not in _FUNCTIONS or not all(issubclass(t, (ndarray, np.ndarray)) for t in types):
            return NotImplemented
        return _FUNCTIONS[func](*args, **kwargs)

    def to_host(self):
        """Synchronize and return an independent NumPy array."""
        return self._backend.download(self)

    def item(self):
        if self.size != 1:
            raise ValueError("item() requires exactly one element")
        return self.to_host().item()

    def astype(self, dtype, *, copy=True):
        dtype = self._backend.validate_dtype(dtype)
        if not copy and dtype == self.dtype:
            return self
        data = self._backend.elementwise("cast", [self], self.shape, dtype)
        return self._wrap(data, self.shape, dtype, self._backend)

    def reshape(self, *shape, order="C"):
        if len(shape) == 1 and not isinstance(shape[0], (int, np.integer)):
            shape = shape[0]
        return reshape(self, shape, order=order)

    # src/openpacho/_array.py:84-86, 145-160
    @property
    def T(self):
        return transpose(self)

    def transpose(self, *axes):
        if len(axes) == 1 and (axes[0] is None or isinstance(axes[0], (tuple, list))):
            axes = axes[0]
        return transpose(self, axes or None)

    def sum(self, axis=None, dtype=None, out=None, keepdims=False):
        return sum(self, axis=axis, dtype=dtype, out=out, keepdims=keepdims)

    def mean(self, axis=None, dtype=None, out=None, keepdims=False):
        return mean(self, axis=axis, dtype=dtype, out=out, keepdims=keepdims)

    def min(self, axis=None, out=None, keepdims=False, initial=None, where=None):
        return amin(self, axis, out, keepdims, _UNSET if initial is None else initial,
                    _UNSET if where is None else where)

    def max(self, axis=None, out=None, keepdims=False, initial=None, where=None):
        return amax(self, axis, out, keepdims, _UNSET if initial is None else initial,
                    _UNSET if where is None else where)


def array(obj, dtype=None, *, copy=True, order="C", backend=None):
    if order != "C":
        raise NotImplementedError("Only C order is supported")
    if isinstance(obj, ndarray):
        target = obj._backend if backend is None else get_backend(backend)
        if target is not obj._backend:
            raise _exc.BackendMismatchError("Use to_backend(a, backend) to transfer explicitly")
        return obj.astype(dtype or obj.dtype, copy=copy)
    target = get_backend(backend)
    host = np.asarray(obj, dtype=dtype, order="C")
    target.validate_dtype(host.dtype)
    return ndarray._wrap(target.upload(host), host.shape, host.dtype, target)


def asarray(obj, dtype=None, *, order="C", backend=None):
    return array(obj, dtype=dtype, copy=False, order=order, backend=backend)


def asnumpy(a):
    return a.to_host() if isinstance(a, ndarray) else np.array(a, copy=True)


def to_backend(a, backend, *, device=None):
    target = get_backend(backend, device=device)
    if isinstance(a, ndarray) and a._backend is target:
        return a
    return asarray(asnumpy(a), backend=target)


def empty(shape, dtype=float, *, order="C", backend=None):
    if order != "C":
        raise NotImplementedError("Only C order is supported")
    shape = _shape(shape)
    target = get_backend(backend)
    dtype = target.validate_dtype(dtype)
    return ndarray._wrap(target.empty(shape, dtype), shape, dtype, target)


def full(shape, fill_value, dtype=None, *, order="C", backend=None):
    if np.ndim(fill_value) != 0:
        raise NotImplementedError("full() supports scalar fill values")
    if order != "C":
        raise NotImplementedError("Only C order is supported")
    shape = _shape(shape)
    target = get_backend(backend)
    dtype = target.validate_dtype(dtype or np.asarray(fill_value).dtype)
    return ndarray._wrap(target.full(shape, fill_value, dtype), shape, dtype, target)


def zeros(shape, dtype=float, *, order="C", backend=None):
    return full(shape, 0, dtype=dtype, order=order, backend=backend)


def ones(shape, dtype=float, *, order="C", backend=None):
    return full(shape, 1, dtype=dtype, order=order, backend=backend)


def reshape(a, shape, order="C"):
    a = asarray(a)
    if order != "C":
        raise NotImplementedError("Only C order is supported")
    shape = (shape,) if isinstance(shape, (int, np.integer)) else tuple(shape)
    shape = tuple(operator.index(d) for d in shape)
    if shape.count(-1) > 1 or any(d < -1 for d in shape):
        raise ValueError("Invalid reshape dimensions")
    if -1 in shape:
        known = prod(d for d in shape if d != -1)
        if known == 0 or a.size % known:
            raise ValueError("Cannot infer reshape dimension")
        shape = tuple(a.size // known if d == -1 else d for d in shape)
    if prod(shape) != a.size:
        raise ValueError("Cannot reshape array to requested shape")
    return ndarray._wrap(a._data, shape, a.dtype, a._backend)


def _common_backend(args):
    found = [a._backend for a in args if isinstance(a, ndarray)]
    if found and any(b is not found[0] for b in found):
        raise _exc.BackendMismatchError("Arrays belong to different backends/devices; use to_backend()")
    return found[0] if found else get_backend()


def _validate_padding(value):
    # src/openpacho/_padding.py:13-16
    if not isinstance(value, (bool, np.bool_)):
        raise TypeError("padding must be a boolean")
    return bool(value)


def matmul(a, b, *, padding=False):
    """Matrix product (src/openpacho/_array.py:457-479); ``padding`` is an
    opt-in hint that backends may decline (b200 always declines)."""
    if padding is not False:
        padding = _validate_padding(padding)
    backend = _common_backend((a, b))
    a, b = asarray(a, backend=backend), asarray(b, backend=backend)
    if a.ndim == 0 or b.ndim == 0:
        raise ValueError("matmul requires arrays with at least one dimension")
    if a.shape[-1] != b.shape[-2 if b.ndim > 1 else 0]:
        raise ValueError("matmul inner dimensions do not match")
    dtype = backend.validate_dtype(np.result_type(a.dtype, b.dtype))
    if dtype.kind == "b":
        raise NotImplementedError("Boolean matmul is not supported")
    a, b = a.astype(dtype, copy=False), b.astype(dtype, copy=False)
    batch = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    shape = batch + (() if a.ndim == 1 else (a.shape[-2],)) + (() if b.ndim == 1 else (b.shape[-1],))
    factory = getattr(backend, "prepare_padded_matmul", None) if padding else None
    plan = None if factory is None else factory(a.shape, b.shape, shape, dtype)
    data = backend.matmul(a, b, shape, dtype) if plan is None else plan.run(a, b)
    return ndarray._wrap(data, shape, dtype, backend)


def dot(a, b):
    """src/openpacho/_array.py:482-491: 0-d operands multiply elementwise,
    vectors and matrices go through matmul."""
    if (a.ndim if isinstance(a, ndarray) else np.ndim(a)) == 0 or (
        b.ndim if isinstance(b, ndarray) else np.ndim(b)
    ) == 0:
        return multiply(a, b)
    if (a.ndim if isinstance(a, ndarray) else np.ndim(a)) > 2 or (
        b.ndim if isinstance(b, ndarray) else np.ndim(b)
    ) > 2:
        raise NotImplementedError("Higher-rank dot differs from batched matmul; use @ for batches")
    return matmul(a, b)


def _axis(axis, ndim):
    axis = operator.index(axis)
    if axis < -ndim or axis >= ndim:
        raise ValueError(f"axis {axis} out of bounds for array of dimension {ndim}")
    return axis % ndim


def _axes(axis, ndim):
    """src/openpacho/_array.py:376-386."""
    if axis is None:
        return tuple(range(ndim))
    values = axis if isinstance(axis, tuple) else (axis,)
    if ndim == 0 and not isinstance(axis, tuple) and axis in (0, -1):
        return ()
    values = tuple(_axis(i, ndim) for i in values)
    if len(set(values)) != len(values):
        raise ValueError("duplicate reduction axis")
    return tuple(sorted(values))


# ---------------------------------------------------------- elementwise --

def resolve_elementwise(ufunc, inputs):
    """Per-operand and result dtypes, and the broadcast shape
    (src/openpacho/_ops.py:42-76, without the graph-capture weak types)."""
    if ufunc is np.where:
        branches = [value if type(value) in (bool, int, float, complex)
                     else value.dtype if hasattr(value, "dtype") else np.asarray(value).dtype
                     for value in inputs[1:]]
        dtype = np.result_type(*branches)
        shape = np.broadcast_shapes(*(value.shape if hasattr(value, "shape") else np.shape(value)
                                      for value in inputs))
        return (np.dtype("bool"), dtype, dtype, dtype), shape
    if ufunc not in UFUNCS.values():
        raise NotImplementedError(f"Unsupported elementwise operation {ufunc.__name__}")
    types = tuple(type(a) if type(a) in (int, float, complex)
                  else a.dtype if hasattr(a, "dtype") else np.asarray(a).dtype for a in inputs)
    resolved = ufunc.resolve_dtypes(types + (None,))
    if ufunc is np.power and resolved[-1].kind in "iu":
        raise NotImplementedError("Integer power is not supported; cast to float or multiply explicitly")
    shape = np.broadcast_shapes(*(getattr(a, "shape", ()) for a in inputs))
    return resolved, shape


def _elementwise(ufunc, *inputs):
    """src/openpacho/_array.py:241-258: operands cast to their resolved
    dtypes on the common backend (host scalars uploaded as 0-d arrays)."""
    backend = _common_backend(inputs)
    resolved, shape = resolve_elementwise(ufunc, inputs)
    for dtype in resolved:
        backend.validate_dtype(dtype)
    args = [asarray(a, dtype=dt, backend=backend) for a, dt in zip(inputs, resolved)]
    shape = np.broadcast_shapes(*(a.shape for a in args))
    data = backend.elementwise(ufunc.__name__, args, shape, resolved[-1])
    return ndarray._wrap(data, shape, resolved[-1], backend)


def _unary_or_binary(ufunc):
    def call(*args):
        return _elementwise(ufunc, *args)

    call.__name__ = ufunc.__name__
    return call


globals().update({name: _unary_or_binary(ufunc) for name, ufunc in UFUNCS.items()})
divide = globals()["true_divide"]

_WHERE_MISSING = object()


def where(condition, x=_WHERE_MISSING, y=_WHERE_MISSING):
    """src/openpacho/_array.py:274-281: both branches are evaluated."""
    if x is _WHERE_MISSING and y is _WHERE_MISSING:
        raise NotImplementedError("One-argument where (nonzero indices) is not supported")
    if x is _WHERE_MISSING or y is _WHERE_MISSING:
        raise TypeError("where requires both x and y")
    return _elementwise(np.where, condition, x, y)


# ------------------------------------------------------- reductions, views --

_UNSET = object()


def sum(a, axis=None, dtype=None, out=None, keepdims=False):  # noqa: A001 - NumPy's name
    """src/openpacho/_array.py:389-409."""
    if out is not None:
        raise NotImplementedError("out= is not supported")
    a = asarray(a)
    axes = _axes(axis, a.ndim)
    if dtype is None:
        dtype = (np.dtype("int64") if a.dtype.kind in "bi"
                 else np.dtype("uint64") if a.dtype.kind == "u" else a.dtype)
    dtype = a._backend.validate_dtype(dtype)
    shape = (tuple(1 if i in axes else d for i, d in enumerate(a.shape)) if keepdims
             else tuple(d for i, d in enumerate(a.shape) if i not in axes))
    data = a._backend.reduce(a, axes, keepdims, dtype)
    return ndarray._wrap(data, shape, dtype, a._backend)


def _extreme(a, axis, out, keepdims, initial, where, operation):
    """src/openpacho/_array.py:412-431."""
    if out is not None:
        raise NotImplementedError("out= is not supported")
    if initial is not _UNSET:
        raise NotImplementedError("initial= is not supported")
    if where is not _UNSET:
        raise NotImplementedError("where= is not supported")
    a = asarray(a)
    axes = _axes(axis, a.ndim)
    if prod(a.shape[i] for i in axes) == 0:
        raise ValueError(f"zero-size array to reduction operation {operation} which has no identity")
    shape = (tuple(1 if i in axes else d for i, d in enumerate(a.shape)) if keepdims
             else tuple(d for i, d in enumerate(a.shape) if i not in axes))
    data = a._backend.reduce(a, axes, keepdims, a.dtype, operation=operation)
    return ndarray._wrap(data, shape, a.dtype, a._backend)


def amin(a, axis=None, out=None, keepdims=False, initial=_UNSET, where=_UNSET):
    """Minimum preserving dtype, propagating NaNs and preferring negative zero ties."""
    return _extreme(a, axis, out, keepdims, initial, where, "min")


def amax(a, axis=None, out=None, keepdims=False, initial=_UNSET, where=_UNSET):
    """Maximum preserving dtype, propagating NaNs and preferring positive zero ties."""
    return _extreme(a, axis, out, keepdims, initial, where, "max")


def mean(a, axis=None, dtype=None, out=None, keepdims=False):
    """src/openpacho/_array.py:444-454."""
    a = asarray(a)
    if a.ndim == 0 and axis is not None and not isinstance(axis, tuple):
        raise ValueError("axis out of bounds for scalar mean")
    dtype = np.dtype(dtype or (a.dtype if a.dtype.kind == "f" else np.float64))
    if dtype.kind != "f":
        raise NotImplementedError("mean supports floating point accumulation only")
    axes = _axes(axis, a.ndim)
    count = prod(a.shape[i] for i in axes)
    return sum(a, axis=axis, dtype=dtype, out=out, keepdims=keepdims) / count


def _strides(shape):
    return tuple(prod(shape[i + 1 :]) for i in range(len(shape)))


def transpose(a, axes=None):
    """src/openpacho/_array.py:355-366 (a gather with permuted strides)."""
    a = asarray(a)
    axes = tuple(reversed(range(a.ndim))) if axes is None else tuple(axes)
    if len(axes) != a.ndim:
        raise ValueError("axes don't match array")
    axes = tuple(_axis(i, a.ndim) for i in axes)
    if len(set(axes)) != a.ndim:
        raise ValueError("repeated axis in transpose")
    shape = tuple(a.shape[i] for i in axes)
    strides = tuple(_strides(a.shape)[i] for i in axes)
    data = a._backend.gather(a, shape, 0, strides)
    return ndarray._wrap(data, shape, a.dtype, a._backend)


def diag(a, k=0):
    """src/openpacho/_array.py:494-503 (matrix diagonals only)."""
    a = asarray(a)
    k = operator.index(k)
    if a.ndim != 2:
        raise NotImplementedError("diag currently extracts matrix diagonals only")
    rows, cols = a.shape
    start_row, start_col = max(0, -k), max(0, k)
    length = max(0, min(rows - start_row, cols - start_col))
    data = a._backend.gather(a, (length,), start_row * cols + start_col, (cols + 1,))
    return ndarray._wrap(data, (length,), a.dtype, a._backend)


def zeros_like(a, dtype=None):
    a = asarray(a)
    return zeros(a.shape, dtype=dtype or a.dtype, backend=a._backend)


def ones_like(a, dtype=None):
    a = asarray(a)
    return ones(a.shape, dtype=dtype or a.dtype, backend=a._backend)


for _name in ("reshape", "dot", "sum", "amin", "amax", "mean", "transpose", "diag", "zeros_like",
              "ones_like", "where"):
    _FUNCTIONS[getattr(np, _name)] = globals()[_name]
_FUNCTIONS[np.min] = amin
_FUNCTIONS[np.max] = amax
