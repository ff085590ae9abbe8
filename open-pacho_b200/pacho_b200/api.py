"""OpenPacho's public array API for the linear-algebra path, over b200.

A self-contained mirror of the parts of OpenPacho's front end that reach the
hot path, with the same names, argument meaning and errors:

* ``ndarray`` -- C-contiguous array owned by one backend
  (src/openpacho/_array.py:31-199), with ``@`` through ``__array_ufunc__``
  (:104-114) and ``np.dot``/``np.linalg.norm`` through ``__array_function__``;
* ``array``/``asarray``/``asnumpy``/``to_backend``/``empty``/``full``/
  ``zeros``/``ones`` (:205-319), ``reshape`` (:337-352);
* ``matmul(a, b, *, padding=False)`` and ``dot`` (:457-491);
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
        return NotImplemented

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
    if sum(d == -1 for d in shape) > 1 or any(d < -1 for d in shape):
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
    """src/openpacho/_array.py:482-491 (0-d operands need elementwise multiply,
    which is outside this backend's path)."""
    if (a.ndim if isinstance(a, ndarray) else np.ndim(a)) == 0 or (
        b.ndim if isinstance(b, ndarray) else np.ndim(b)
    ) == 0:
        raise NotImplementedError("0-d dot is an elementwise multiply; not on the b200 path")
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


for _name in ("reshape", "dot"):
    _FUNCTIONS[getattr(np, _name)] = globals()[_name]
