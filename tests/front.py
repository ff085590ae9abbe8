"""A small array type for the GPU tests (test code, not part of the product).

The product is a backend: OpenPacho's own front end (``openpacho.asarray``,
``@``, ``linalg.norm`` ...) drives ``B200Backend`` once ``pacho_b200.register()``
has run.  OpenPacho itself is not installed on the GPU machines, so the GPU
tests drive the same backend calls through this module instead.  It makes
the calls the front end makes, with the same shape and dtype rules
(NumPy's: broadcasting, ``np.result_type`` for matmul, the ufunc's own type
resolution with Python scalars as weak types), and nothing else:

  asarray/asnumpy      upload / download
  a @ b, matmul, dot   backend.matmul(a, b, out_shape, dtype)
  linalg.norm          backend.norm(x, axes, keepdims, dtype)
  ufuncs, operators    operands cast to the resolved dtypes, then
                       backend.elementwise(name, operands, shape, dtype)
  sum/amin/amax/mean   backend.reduce
  transpose, diag      backend.gather
"""

from __future__ import annotations

from math import prod
from types import SimpleNamespace

import numpy as np

PY_SCALARS = (bool, int, float)


class Scalar:
    """A host scalar operand (the backend uploads it as one element)."""

    _host_scalar = True
    shape = ()
    ndim = 0

    def __init__(self, value, dtype):
        self.dtype = np.dtype(dtype)
        self._data = np.asarray(value, dtype=self.dtype)[()]


class Arr:
    """Device array: backend, storage and (shape, dtype)."""

    __array_priority__ = 100

    def __init__(self, backend, data, shape, dtype):
        self._backend, self._data = backend, data
        self.shape, self.dtype = tuple(int(d) for d in shape), np.dtype(dtype)

    ndim = property(lambda self: len(self.shape))
    size = property(lambda self: prod(self.shape))

    def numpy(self):
        return self._backend.download(self)

    def item(self):
        return self.numpy().reshape(()).item() if self.size == 1 else self.numpy().item()

    def astype(self, dtype):
        dtype = np.dtype(dtype)
        if dtype == self.dtype:
            return self
        return Arr(self._backend, self._backend.elementwise("cast", [self], self.shape, dtype),
                   self.shape, dtype)

    # NumPy ufuncs on these arrays run on the backend.
    def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
        if method != "__call__" or kwargs:
            return NotImplemented
        if ufunc is np.matmul:
            return matmul(*inputs)
        return apply(ufunc.__name__, *inputs)

    def __matmul__(self, other):
        return matmul(self, other)

    def __rmatmul__(self, other):
        return matmul(other, self)


def _binary(name, reflected=False):
    if reflected:
        return lambda self, other: apply(name, other, self)
    return lambda self, other: apply(name, self, other)


for _op, _name in (("add", "add"), ("sub", "subtract"), ("mul", "multiply"), ("truediv", "true_divide"),
                   ("pow", "power")):
    setattr(Arr, f"__{_op}__", _binary(_name))
    setattr(Arr, f"__r{_op}__", _binary(_name, True))
for _op, _name in (("eq", "equal"), ("ne", "not_equal"), ("lt", "less"), ("le", "less_equal"),
                   ("gt", "greater"), ("ge", "greater_equal")):
    setattr(Arr, f"__{_op}__", _binary(_name))
Arr.__neg__ = lambda self: apply("negative", self)
Arr.__pos__ = lambda self: apply("positive", self)
Arr.__abs__ = lambda self: apply("absolute", self)
Arr.__hash__ = object.__hash__


def wrap(data, shape, dtype, backend):
    return Arr(backend, data, shape, dtype)


def asarray(x, backend=None):
    if isinstance(x, Arr):
        return x
    host = np.asarray(x, order="C")  # keeps 0-d arrays 0-d (ascontiguousarray would not)
    return Arr(backend, backend.upload(host), host.shape, host.dtype)


def asnumpy(a):
    return a.numpy()


def _backend_of(values):
    for v in values:
        if isinstance(v, Arr):
            return v._backend
    raise TypeError("no device array among the operands")


def apply(name, *inputs):
    """One elementwise operation with NumPy's type resolution."""
    backend = _backend_of(inputs)
    if name == "where":
        samples = [v if isinstance(v, PY_SCALARS) else np.empty(0, v.dtype) for v in inputs[1:]]
        out = np.result_type(*samples)
        resolved = (np.dtype(bool), out, out, out)
    else:
        types = tuple(np.dtype(bool) if isinstance(v, bool) else type(v) if isinstance(v, PY_SCALARS)
                      else v.dtype for v in inputs)
        resolved = tuple(np.dtype(t) for t in getattr(np, name).resolve_dtypes(types + (None,)))
    shape = np.broadcast_shapes(*(getattr(v, "shape", ()) for v in inputs))
    operands = []
    for v, dt in zip(inputs, resolved):
        if isinstance(v, PY_SCALARS):
            operands.append(Scalar(v, dt))
        else:
            operands.append(asarray(v, backend).astype(dt))
    dtype = resolved[-1]
    return Arr(backend, backend.elementwise(name, operands, shape, dtype), shape, dtype)


def _ufunc(name):
    return lambda *inputs: apply(name, *inputs)


for _name in ("add", "subtract", "multiply", "true_divide", "power", "negative", "positive", "absolute",
              "sqrt", "exp", "log", "sin", "cos", "tanh", "equal", "not_equal", "less", "less_equal",
              "greater", "greater_equal", "isfinite"):
    globals()[_name] = _ufunc(_name)


def where(cond, x, y):
    return apply("where", cond, x, y)


def matmul(a, b):
    backend = _backend_of((a, b))
    a, b = asarray(a, backend), asarray(b, backend)
    dtype = np.result_type(a.dtype, b.dtype)
    a, b = a.astype(dtype), b.astype(dtype)
    batch = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    shape = batch + (() if a.ndim == 1 else (a.shape[-2],)) + (() if b.ndim == 1 else (b.shape[-1],))
    return Arr(backend, backend.matmul(a, b, shape, dtype), shape, dtype)


def dot(a, b):
    return matmul(a, b)


def _axes(axis, ndim):
    if axis is None:
        return tuple(range(ndim))
    values = axis if isinstance(axis, tuple) else (axis,)
    return tuple(sorted(int(i) % ndim for i in values))


def _kept(shape, axes, keepdims):
    if keepdims:
        return tuple(1 if i in axes else d for i, d in enumerate(shape))
    return tuple(d for i, d in enumerate(shape) if i not in axes)


def _norm(x, axis=None, keepdims=False):
    if isinstance(axis, tuple) and len(axis) not in (1, 2):
        raise ValueError("norm takes one vector axis or two matrix axes")
    if x.dtype.kind != "f":
        x = x.astype(np.float64)
    axes = _axes(axis, x.ndim)
    shape = _kept(x.shape, axes, keepdims)
    return Arr(x._backend, x._backend.norm(x, axes, keepdims, x.dtype), shape, x.dtype)


linalg = SimpleNamespace(norm=_norm)


def _reduce(a, axis, dtype, keepdims, operation):
    axes = _axes(axis, a.ndim)
    dtype = np.dtype(dtype or a.dtype)
    shape = _kept(a.shape, axes, keepdims)
    data = a._backend.reduce(a, axes, keepdims, dtype, operation=operation)
    return Arr(a._backend, data, shape, dtype)


def sum(a, axis=None, dtype=None, keepdims=False):  # noqa: A001 - NumPy's name
    return _reduce(a, axis, dtype, keepdims, "sum")


def amin(a, axis=None, keepdims=False):
    return _reduce(a, axis, None, keepdims, "min")


def amax(a, axis=None, keepdims=False):
    return _reduce(a, axis, None, keepdims, "max")


def mean(a, axis=None, keepdims=False):
    dtype = a.dtype if a.dtype.kind == "f" else np.dtype(np.float64)
    count = prod(a.shape[i] for i in _axes(axis, a.ndim))
    return sum(a, axis=axis, dtype=dtype, keepdims=keepdims) / count


def _strides(shape):
    out, step = [], 1
    for d in reversed(shape):
        out.append(step)
        step *= d
    return tuple(reversed(out))


def transpose(a, axes=None):
    axes = tuple(reversed(range(a.ndim))) if axes is None else tuple(axes)
    own = _strides(a.shape)
    shape = tuple(a.shape[i] for i in axes)
    data = a._backend.gather(a, shape, 0, tuple(own[i] for i in axes))
    return Arr(a._backend, data, shape, a.dtype)


def diag(a, k=0):
    rows, cols = a.shape
    start = (0, k) if k >= 0 else (-k, 0)
    n = max(0, min(rows - start[0], cols - start[1]))
    data = a._backend.gather(a, (n,), start[0] * cols + start[1], (cols + 1,))
    return Arr(a._backend, data, (n,), a.dtype)


def zeros(shape, dtype, backend):
    return Arr(backend, backend.full(shape, 0, dtype), shape, dtype)


def full(shape, value, dtype, backend):
    return Arr(backend, backend.full(shape, value, dtype), shape, dtype)
