"""A host stand-in for ``B200Backend`` (CPU tests of the plumbing only).

``HostB200`` answers the backend protocol with the NumPy-backend oracle on host
arrays, so OpenPacho's real front end (``asarray``, ``@``, ``linalg.norm``,
``compile`` with this package's lowering, the ``pacho`` command) can run
end to end on a machine without a GPU, and so a test can record the exact
protocol calls the front end makes.  It is an ``B200Backend`` subclass, so
``register()`` and OpenPacho's dispatch treat it as the b200 backend; only the
storage and the arithmetic differ.  Nothing in the product imports it.
"""

from __future__ import annotations

import threading
from math import prod

import numpy as np

from oracle import numpy_backend
from pacho_b200.backend import B200Backend


class HostBuffer:
    """Flat host storage in place of a DeviceBuffer (same ``backend`` link)."""

    __slots__ = ("array", "backend", "__weakref__")

    def __init__(self, array, backend):
        self.array = np.ascontiguousarray(array).reshape(-1)
        self.backend = backend

    @property
    def nbytes(self):
        return self.array.nbytes


def _value(a):
    """Host value of a protocol operand (array or host scalar)."""
    if getattr(a, "_host_scalar", False):
        return np.asarray(a._data, dtype=a.dtype)
    return a._data.array.reshape(a.shape)


class HostB200(B200Backend):
    name = "b200"
    fp64 = True

    def __init__(self, device="host stand-in"):  # no library, no GPU
        self.device = device
        self.ordinal = 0
        self._lock = threading.RLock()
        self._closed = False
        self.calls = []

    def _log(self, method, *details):
        self.calls.append((method,) + details)

    def _buffer(self, array):
        return HostBuffer(array, self)

    def __del__(self):
        pass

    def close(self):
        self._closed = True

    def synchronize(self):
        self._log("synchronize")

    def upload(self, a):
        host = np.array(a, copy=True)
        self.validate_dtype(host.dtype)
        self._log("upload", host.shape, host.dtype)
        return self._buffer(host)

    def download(self, a):
        self._log("download", tuple(a.shape), np.dtype(a.dtype))
        return _value(a).copy()

    def empty(self, shape, dtype):
        dtype = self.validate_dtype(dtype)
        return self._buffer(np.zeros(prod(shape), dtype))

    def full(self, shape, value, dtype):
        dtype = self.validate_dtype(dtype)
        self._log("full", tuple(shape), value, dtype)
        return self._buffer(np.full(prod(shape), value, dtype))

    def matmul(self, a, b, shape, dtype):
        self._log("matmul", tuple(a.shape), tuple(b.shape), tuple(shape), np.dtype(dtype))
        with np.errstate(all="ignore"):
            out = numpy_backend.matmul(_value(a), _value(b))
        return self._buffer(np.asarray(out, dtype).reshape(shape))

    def norm(self, a, axes, keepdims, dtype):
        self._log("norm", tuple(a.shape), tuple(axes), keepdims, np.dtype(dtype))
        return self._buffer(numpy_backend.norm_data(_value(a), tuple(axes), dtype))

    def elementwise(self, name, args, shape, dtype):
        self._log("elementwise", name, tuple(tuple(a.shape) for a in args), tuple(shape), np.dtype(dtype))
        out = numpy_backend.elementwise(name, [_value(a) for a in args], dtype)
        return self._buffer(np.broadcast_to(out, tuple(shape)))

    def gather(self, a, shape, offset, strides):
        self._log("gather", tuple(a.shape), tuple(shape), offset, tuple(strides))
        return self._buffer(numpy_backend.gather(_value(a), tuple(shape), offset, tuple(strides)))

    def reduce(self, a, axes, keepdims, dtype, *, operation="sum"):
        self._log("reduce", tuple(a.shape), tuple(axes), keepdims, np.dtype(dtype), operation)
        return self._buffer(numpy_backend.reduce(_value(a), tuple(axes), False, dtype, operation))

    def residual_matvec(self, a, x, b):
        self._log("residual_matvec", tuple(a.shape), tuple(x.shape), tuple(b.shape))
        y = numpy_backend.matmul(_value(a), _value(x))
        return self._buffer(numpy_backend.elementwise("subtract", (_value(b), y), b.dtype))

    def release_cached_memory(self):
        self._log("release_cached_memory")
