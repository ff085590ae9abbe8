"""``B200Backend``: OpenPacho's backend protocol implemented on libpacho_b200.

The object plugs in where OpenPacho's ``NumpyBackend``/``CUDABackend`` do
(src/openpacho/backends.py:82-150, src/openpacho/_cuda.py:129-679): the
front end calls ``validate_dtype``, ``upload``, ``download``, ``empty``,
``full``, ``matmul(a, b, shape, dtype)``, ``norm(a, axes, keepdims, dtype)``
and ``synchronize`` with operands that expose ``shape``, ``ndim``, ``dtype``
and ``_data``; around the path, ``elementwise``, ``gather`` and ``reduce``
(astype, solver arithmetic, sum/mean/min/max, transpose/diag).  Storage is a
:class:`DeviceBuffer` (flat, C-contiguous).  Unsupported requests raise
``NotImplementedError``; nothing ever runs on the host CPU instead.
"""

from __future__ import annotations

import ctypes as C
import threading
import weakref
from contextlib import contextmanager
from math import prod

import numpy as np

from . import _lib, pool
from . import exceptions as _exc

SUPPORTED = (np.dtype(np.float32), np.dtype(np.float64), np.dtype(np.bool_))
MAX_DIMS = 8  # per operand, for elementwise / gather / reduce


class DeviceBuffer:
    """Flat device allocation owned by one backend (cf. ``_Allocation``,
    src/openpacho/_cuda.py:100-126).  Freed stream-ordered when collected."""

    __slots__ = ("backend", "ptr", "nbytes", "__weakref__")

    def __init__(self, backend: "B200Backend", ptr: int, nbytes: int):
        self.backend = backend
        self.ptr = ptr
        self.nbytes = nbytes

    def __int__(self):
        return self.ptr

    def release(self):
        ptr, self.ptr = self.ptr, 0
        backend = self.backend
        if ptr and backend is not None and not backend._closed:
            with backend._lock:
                backend._lib.pb_free(backend._ctx, 0, C.c_void_p(ptr))

    def __del__(self):
        try:
            self.release()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class DeviceArray:
    """A typed view of one :class:`DeviceBuffer`: the four attributes the
    backend protocol reads of an operand (``shape``, ``ndim``, ``dtype``,
    ``_data``) plus ``numpy()``.  It is what this package's own functions
    (multi-GPU, the compiled-plan lowering) return when they are not handed
    OpenPacho arrays; it has no arithmetic of its own -- OpenPacho's
    ``ndarray`` is the array type users compute with."""

    __slots__ = ("_backend", "_data", "shape", "dtype")

    def __init__(self, backend: "B200Backend", data: DeviceBuffer, shape, dtype):
        self._backend = backend
        self._data = data
        self.shape = tuple(int(d) for d in shape)
        self.dtype = np.dtype(dtype)

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def size(self) -> int:
        return prod(self.shape)

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    def numpy(self) -> np.ndarray:
        return self._backend.download(self)

    def item(self):
        if self.size != 1:
            raise ValueError("only one-element arrays convert to a Python scalar")
        return self.numpy().reshape(()).item()

    def __repr__(self):
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype}, device={self._backend.ordinal})"


class Graph:
    """A captured sequence of library calls (``B200Backend.capture``),
    replayed on the device stream by ``launch()``; ``close()`` frees it."""

    def __init__(self, backend: "B200Backend", handle: int, launches: int):
        self._backend, self._handle, self.launches = backend, handle, launches

    def launch(self):
        b = self._backend
        with b._lock:
            b._require_open()
            if not self._handle:
                raise RuntimeError("graph is closed")
            b._check(b._lib.pb_graph_launch(b._ctx, 0, C.c_void_p(self._handle)), "pb_graph_launch")

    def close(self):
        b, h = self._backend, self._handle
        self._handle = 0
        if h and not b._closed:
            with b._lock:
                b._check(b._lib.pb_graph_destroy(b._ctx, 0, C.c_void_p(h)), "pb_graph_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def wrap_like(template, data, shape, dtype, backend):
    """An array of ``template``'s kind around ``data``: OpenPacho's ndarray
    (its ``_wrap`` constructor, src/openpacho/_array.py:43-51) when the caller
    passed OpenPacho arrays, else a :class:`DeviceArray`."""
    wrap = getattr(type(template), "_wrap", None)
    if wrap is not None:
        return wrap(data, tuple(shape), np.dtype(dtype), backend)
    return DeviceArray(backend, data, shape, dtype)


def _broadcast_strides(shape, own):
    """Element strides of a C-contiguous operand of shape ``own`` seen through
    NumPy broadcasting to ``shape`` (0 along broadcast dimensions)."""
    padded = (1,) * (len(shape) - len(own)) + tuple(own)
    strides, step = [0] * len(shape), 1
    for d in range(len(shape) - 1, -1, -1):
        strides[d] = 0 if padded[d] == 1 and shape[d] != 1 else step
        step *= padded[d]
    return strides


def _matrix_strides(batch, own):
    """Per broadcast batch dim, the stride in whole matrices of an operand
    whose own batch shape is ``own`` (0 where the operand broadcasts)."""
    padded = (1,) * (len(batch) - len(own)) + tuple(own)
    strides = []
    for j, dim in enumerate(padded):
        strides.append(0 if dim == 1 else prod(padded[j + 1 :]))
    return strides


class B200Backend:
    """OpenPacho backend object for one B200 GPU (the ``"b200"`` name)."""

    name = "b200"
    fp64 = True
    # One GPU unless the context holds several (set in __init__).
    ordinals = (0,)
    _pool = None
    split_min_gain = pool.MIN_GAIN

    def __init__(self, device=None, *, gpus=None):
        self._lib = _lib.load()
        try:
            ordinals = pool.parse_devices(device, gpus)
        except ValueError as exc:
            raise _exc.BackendUnavailableError(str(exc)) from exc
        identifier = ordinals[0]
        count = C.c_int(0)
        status = self._lib.pb_device_count(C.byref(count))
        if status != _lib.PB_OK or count.value == 0:
            raise _exc.BackendUnavailableError(f"no CUDA device for b200: {_lib.last_error()}")
        missing = [o for o in ordinals if not 0 <= o < count.value]
        if missing:
            raise _exc.BackendUnavailableError(f"b200 device {device!r} not found ({count.value} visible)")
        name = C.create_string_buffer(256)
        total = C.c_size_t(0)
        sms, major, minor = C.c_int(), C.c_int(), C.c_int()
        _lib.check(
            self._lib.pb_device_info(identifier, name, 256, C.byref(total), C.byref(sms),
                                     C.byref(major), C.byref(minor)),
            "pb_device_info",
        )
        self.ordinal = identifier
        self.device = name.value.decode()
        self.memory_bytes = total.value
        self.sm_count = sms.value
        self.compute_capability = (major.value, minor.value)
        self._lock = threading.RLock()
        self._closed = False
        self._buffers = weakref.WeakSet()
        self._graphs = weakref.WeakSet()
        ctx = C.c_void_p()
        status = self._lib.pb_init(len(ordinals), (C.c_int * len(ordinals))(*ordinals), C.byref(ctx))
        if status != _lib.PB_OK:
            raise _exc.BackendUnavailableError(f"b200 initialization failed: {_lib.last_error()}")
        self._ctx = ctx
        # Arrays live on the first GPU; with more, large products are split.
        self.ordinals = tuple(ordinals)
        self._pool = pool.DevicePool(self, len(ordinals)) if len(ordinals) > 1 else None

    # ---------------------------------------------------------------- basics
    def __repr__(self):
        if len(self.ordinals) > 1:
            return f"B200Backend(devices={list(self.ordinals)}, name={self.device!r})"
        return f"B200Backend(device={self.ordinal}, name={self.device!r})"

    def _check(self, status, what):
        _lib.check(status, what)

    def _require_open(self):
        if self._closed:
            raise RuntimeError("b200 backend is closed")

    def validate_dtype(self, dtype):
        """bool, float32 and float64, as the reference CUDA backend
        (src/openpacho/_cuda.py:226-230); matmul and norm take the floats."""
        try:
            dtype = np.dtype(dtype)
        except TypeError as exc:
            raise _exc.UnsupportedDtypeError(str(exc)) from exc
        if dtype not in SUPPORTED or not dtype.isnative:
            raise _exc.UnsupportedDtypeError(
                f"b200 backend supports bool, float32 and float64, not {dtype}")
        return dtype

    @contextmanager
    def execution_scope(self):
        with self._lock:
            self._require_open()
            yield

    def synchronize(self):
        with self._lock:
            self._require_open()
            self._check(self._lib.pb_sync(self._ctx, 0), "pb_sync")

    # ---------------------------------------------------------------- memory
    def _alloc(self, nbytes):
        ptr = C.c_void_p()
        with self._lock:
            self._require_open()
            self._check(self._lib.pb_alloc(self._ctx, 0, max(int(nbytes), 1), C.byref(ptr)),
                        "pb_alloc")
        buf = DeviceBuffer(self, ptr.value, int(nbytes))
        self._buffers.add(buf)
        return buf

    def empty(self, shape, dtype):
        dtype = self.validate_dtype(dtype)
        return self._alloc(prod(shape) * dtype.itemsize)

    def full(self, shape, value, dtype):
        dtype = self.validate_dtype(dtype)
        out = self.empty(shape, dtype)
        count = prod(shape)
        if count:
            with self._lock:
                self._check(
                    self._lib.pb_fill(self._ctx, 0, _lib.dtype_code(dtype), C.c_void_p(out.ptr),
                                      count, float(np.asarray(value, dtype=dtype))),
                    "pb_fill",
                )
        return out

    def upload(self, a):
        """Synchronous copy: the device buffer snapshots the host array."""
        host = np.ascontiguousarray(a)
        self.validate_dtype(host.dtype)
        out = self._alloc(host.nbytes)
        if host.nbytes:
            with self._lock:
                self._check(
                    self._lib.pb_h2d(self._ctx, 0, C.c_void_p(out.ptr),
                                     C.c_void_p(host.ctypes.data), host.nbytes, 1),
                    "pb_h2d",
                )
        return out

    def download(self, a):
        out = np.empty(a.shape, a.dtype)
        with self._lock:
            self._require_open()
            self._check(
                self._lib.pb_d2h(self._ctx, 0, C.c_void_p(out.ctypes.data),
                                 C.c_void_p(a._data.ptr), out.nbytes),
                "pb_d2h",
            )
        return out

    def release_cached_memory(self):
        with self._lock:
            self._require_open()
            self._check(self._lib.pb_trim(self._ctx, 0), "pb_trim")

    # ------------------------------------------------------------ hot path
    def matmul(self, a, b, shape, dtype):
        """``a @ b`` with NumPy broadcasting of leading dimensions.

        Mirrors the shape handling of CUDABackend.matmul
        (src/openpacho/_cuda.py:493-517): vector-vector is a DOT, a trailing
        vector is a GEMV over the flattened rows of ``a``, everything else one
        batched GEMM launch with per-operand batch strides (0 = broadcast)."""
        dtype = self.validate_dtype(dtype)
        if dtype.kind != "f":
            raise NotImplementedError("b200 matmul requires float32 or float64")
        if a.dtype != dtype or b.dtype != dtype:
            raise NotImplementedError("b200 matmul needs operands already in the result dtype")
        code = _lib.dtype_code(dtype)
        m, k = (1, a.shape[0]) if a.ndim == 1 else a.shape[-2:]
        n = b.shape[-1] if b.ndim > 1 else 1
        out = self.empty(shape, dtype)
        if not prod(shape):
            return out
        with self._lock:
            self._require_open()
            ctx, lib = self._ctx, self._lib
            A, B, O = C.c_void_p(a._data.ptr), C.c_void_p(b._data.ptr), C.c_void_p(out.ptr)
            if a.ndim == 1 and b.ndim == 1:
                self._check(lib.pb_dot(ctx, 0, code, k, A, B, O), "pb_dot")
            elif b.ndim == 1:
                rows = prod(a.shape[:-1])
                self._check(lib.pb_gemv(ctx, 0, code, rows, k, A, B, O), "pb_gemv")
            else:
                a_batch = a.shape[:-2] if a.ndim > 1 else ()
                b_batch = b.shape[:-2]
                batch = np.broadcast_shapes(a_batch, b_batch)
                if self._pool is not None and a.ndim > 1:
                    if self._split_matmul(code, dtype, a, b, batch, m, n, k, A, B, O):
                        return out
                self._check(
                    lib.pb_gemm(ctx, 0, code, len(batch), _lib.i64_array(batch),
                                _lib.i64_array(_matrix_strides(batch, a_batch)),
                                _lib.i64_array(_matrix_strides(batch, b_batch)),
                                m, n, k, A, B, O),
                    "pb_gemm",
                )
        return out

    def matmul_host(self, a, b, *, chunks=0):
        """``a @ b`` for host (NumPy) arrays of at least two dimensions, with
        NumPy's broadcasting of leading dimensions: one ``pb_gemm_host`` call,
        whose upload, product and download overlap piece by piece.  Returns a
        new host array.  Pinned operands (``pb_host_register``) copy
        asynchronously; others through the driver's staging."""
        a = np.ascontiguousarray(a)
        b = np.ascontiguousarray(b)
        if a.ndim < 2 or b.ndim < 2:
            raise ValueError("matmul_host takes operands of at least two dimensions")
        if a.dtype != b.dtype:
            raise NotImplementedError("matmul_host needs operands of one dtype")
        dtype = self.validate_dtype(a.dtype)
        if dtype.kind != "f":
            raise NotImplementedError("b200 matmul requires float32 or float64")
        m, k = a.shape[-2:]
        k2, n = b.shape[-2:]
        if k != k2:
            raise ValueError(f"matmul: inner dimensions differ ({k} and {k2})")
        a_batch, b_batch = a.shape[:-2], b.shape[:-2]
        batch = tuple(np.broadcast_shapes(a_batch, b_batch))
        out = np.empty(batch + (m, n), dtype)
        if not out.size:
            return out
        with self._lock:
            self._require_open()
            self._check(
                self._lib.pb_gemm_host(self._ctx, 0, _lib.dtype_code(dtype), len(batch), _lib.i64_array(batch),
                                       _lib.i64_array(_matrix_strides(batch, a_batch)),
                                       _lib.i64_array(_matrix_strides(batch, b_batch)), m, n, k,
                                       C.c_void_p(a.ctypes.data), C.c_void_p(b.ctypes.data),
                                       C.c_void_p(out.ctypes.data), int(chunks)),
                "pb_gemm_host")
        return out

    def _split_matmul(self, code, dtype, a, b, batch, m, n, k, A, B, O) -> bool:
        """The product over every GPU of the context, when it pays."""
        sp = pool.plan(a.shape, b.shape, batch, m, n, k)
        if sp is None or sp.outer < 2:
            return False
        isz = dtype.itemsize
        flops = 2.0 * prod(batch) * m * n * k
        if not pool.worth_splitting(flops, isz, prod(a.shape) * isz, prod(b.shape) * isz,
                                    prod(batch) * m * n * isz, len(self.ordinals),
                                    min_gain=self.split_min_gain):
            return False
        lib, ctx = self._lib, self._ctx

        def gemm(dev, outer, pa, pb, pc):
            if not sp.batch:
                status = lib.pb_gemm(ctx, dev, code, 0, _lib.i64_array(()), _lib.i64_array(()),
                                     _lib.i64_array(()), outer, n, k, C.c_void_p(pa), C.c_void_p(pb),
                                     C.c_void_p(pc))
            else:
                bshape = (outer,) + sp.batch[1:]
                status = lib.pb_gemm(ctx, dev, code, len(bshape), _lib.i64_array(bshape),
                                     _lib.i64_array(_matrix_strides(bshape, bshape)),
                                     _lib.i64_array(_matrix_strides(bshape, bshape if sp.b_block else ())),
                                     m, n, k, C.c_void_p(pa), C.c_void_p(pb), C.c_void_p(pc))
            self._check(status, "pb_gemm")

        self._pool.matmul(code, isz, sp, A.value, B.value, O.value, gemm)
        return True

    def norm(self, a, axes, keepdims, dtype):
        """Euclidean/Frobenius norm over ``axes`` (norm_data,
        src/openpacho/_norm.py:39-118); ``keepdims`` only shapes the wrapper."""
        dtype = self.validate_dtype(dtype)
        if dtype.kind != "f":
            raise NotImplementedError("b200 norm requires float32 or float64")
        if a.dtype != dtype:
            raise NotImplementedError("b200 norm needs its input in the result dtype")
        code = _lib.dtype_code(dtype)
        shape = tuple(a.shape)
        axes = tuple(sorted(axes))
        count = prod(d for i, d in enumerate(shape) if i not in axes)
        reduced = prod(shape[i] for i in axes)
        out = self.empty((count,), dtype)
        if not count:
            return out
        with self._lock:
            self._require_open()
            X, O = C.c_void_p(a._data.ptr), C.c_void_p(out.ptr)
            if not axes or axes == tuple(range(axes[0], axes[-1] + 1)):
                first = axes[0] if axes else len(shape)
                last = axes[-1] if axes else len(shape) - 1
                outer = prod(shape[:first])
                inner = prod(shape[last + 1 :])
                self._check(
                    self._lib.pb_norm(self._ctx, 0, code, outer, reduced, inner, X, O), "pb_norm"
                )
            else:
                elem = [prod(shape[i + 1 :]) for i in range(len(shape))]
                keep = [i for i in range(len(shape)) if i not in axes]
                self._check(
                    self._lib.pb_norm_strided(
                        self._ctx, 0, code, len(keep), _lib.i64_array(shape[i] for i in keep),
                        _lib.i64_array(elem[i] for i in keep), len(axes),
                        _lib.i64_array(shape[i] for i in axes),
                        _lib.i64_array(elem[i] for i in axes), X, O),
                    "pb_norm_strided",
                )
        return out

    def residual_matvec(self, a, x, b):
        """``b - a @ x`` in one GEMV launch with the subtraction in its
        epilogue (``pb_gemv_residual``); the compiled plans call it for a
        residual whose product has no other use (src/openpacho/_compiler.py:
        157-176, 306-307).  Checks as residual_matvec_data
        (src/openpacho/_gemv.py:10-23)."""
        if a.ndim != 2 or x.ndim != 1 or b.ndim != 1:
            raise ValueError("Residual GEMV requires a matrix and two vectors")
        rows, columns = a.shape
        if tuple(x.shape) != (columns,) or tuple(b.shape) != (rows,):
            raise ValueError("Residual GEMV dimensions do not match")
        dtype = np.dtype(a.dtype)
        if dtype not in (np.dtype(np.float32), np.dtype(np.float64)) or x.dtype != dtype or b.dtype != dtype:
            raise ValueError("Residual GEMV requires matching float32/float64 dtypes")
        if any(getattr(v._data, "backend", None) is not self for v in (a, x, b)):
            raise ValueError("Residual GEMV inputs must belong to the same backend")
        out = self.empty((rows,), dtype)
        if rows:
            with self._lock:
                self._require_open()
                self._check(
                    self._lib.pb_gemv_residual(self._ctx, 0, _lib.dtype_code(dtype), rows, columns,
                                               C.c_void_p(a._data.ptr), C.c_void_p(x._data.ptr),
                                               C.c_void_p(b._data.ptr), C.c_void_p(out.ptr)),
                    "pb_gemv_residual",
                )
        return out

    def create_lowering(self):
        """The compiled-plan lowering (src/openpacho/_lowering.py:224-231):
        residual GEMVs fused into the GEMV epilogue, elementwise groups and
        their reductions on the b200 kernels."""
        from .lowering import B200Lowering

        return B200Lowering(self)

    def prepare_padded_matmul(self, ashape, bshape, shape, dtype):
        """Decline the padding hint (src/openpacho/_padding.py:19-22): TMA
        zero-fills ragged tiles, so padded copies would only add traffic."""
        return None

    # ------------------------------------------------------ around the path
    def elementwise(self, name, args, shape, dtype):
        """``name`` over broadcast operands into a new ``shape`` array of
        ``dtype`` (CUDABackend.elementwise, src/openpacho/_cuda.py:416-434;
        operation names of _EXPRESSIONS, :21-46).  Operands are arrays of
        this backend, or host scalars (``_host_scalar``), uploaded once."""
        dtype = self.validate_dtype(dtype)
        op = _lib.EW_OPS.get(name)
        if op is None:
            raise NotImplementedError(f"b200 elementwise has no operation {name!r}")
        shape = tuple(int(d) for d in shape)
        if len(shape) > MAX_DIMS:
            raise NotImplementedError(f"b200 elementwise supports at most {MAX_DIMS} dimensions")
        out = self.empty(shape, dtype)
        if not prod(shape):
            return out
        ptrs, codes, strides, keep = [], [], [], []
        for a in args:
            if getattr(a, "_host_scalar", False):
                data = self.upload(np.asarray(a._data, dtype=a.dtype).reshape(1))
                keep.append(data)
                own = ()
            else:
                data, own = a._data, tuple(a.shape)
            ptrs.append(data.ptr)
            codes.append(_lib.dtype_code(a.dtype))
            strides.extend(_broadcast_strides(shape, own))
        with self._lock:
            self._require_open()
            self._check(
                self._lib.pb_elementwise(
                    self._ctx, 0, op, len(args), (C.c_void_p * len(ptrs))(*ptrs),
                    (C.c_int * len(codes))(*codes), _lib.i64_array(strides), len(shape),
                    _lib.i64_array(shape), _lib.dtype_code(dtype), C.c_void_p(out.ptr)),
                f"pb_elementwise({name})",
            )
        return out

    def gather(self, a, shape, offset, strides):
        """Strided copy out of ``a``'s flat storage (CUDABackend.gather,
        src/openpacho/_cuda.py:436-447): element offset and strides."""
        shape = tuple(int(d) for d in shape)
        if len(shape) > MAX_DIMS:
            raise NotImplementedError(f"b200 gather supports at most {MAX_DIMS} dimensions")
        out = self.empty(shape, a.dtype)
        if not prod(shape):
            return out
        with self._lock:
            self._require_open()
            self._check(
                self._lib.pb_gather(self._ctx, 0, _lib.dtype_code(a.dtype), C.c_void_p(a._data.ptr),
                                    len(shape), _lib.i64_array(shape), int(offset),
                                    _lib.i64_array(int(s) for s in strides), C.c_void_p(out.ptr)),
                "pb_gather",
            )
        return out

    def reduce(self, a, axes, keepdims, dtype, *, operation="sum"):
        """sum/min/max over ``axes`` into ``prod(kept)`` values of ``dtype``
        (CUDABackend.reduce, src/openpacho/_cuda.py:449-492)."""
        dtype = self.validate_dtype(dtype)
        if operation not in _lib.REDUCE_OPS:
            raise ValueError(f"Unknown reduction operation: {operation}")
        if dtype.kind == "b" and operation == "sum":
            raise NotImplementedError("Boolean reduction is not implemented on b200")
        shape = tuple(a.shape)
        if len(shape) > MAX_DIMS:
            raise NotImplementedError(f"b200 reduce supports at most {MAX_DIMS} dimensions")
        axes = tuple(sorted(axes))
        count = prod(d for i, d in enumerate(shape) if i not in axes)
        out = self.empty((count,), dtype)
        if not count:
            return out
        mask = 0
        for i in axes:
            mask |= 1 << i
        with self._lock:
            self._require_open()
            self._check(
                self._lib.pb_reduce(self._ctx, 0, _lib.REDUCE_OPS[operation], _lib.dtype_code(a.dtype),
                                    C.c_void_p(a._data.ptr), len(shape), _lib.i64_array(shape), mask,
                                    _lib.dtype_code(dtype), C.c_void_p(out.ptr)),
                f"pb_reduce({operation})",
            )
        return out

    # --------------------------------------------------------------- graphs
    def capture(self, fn) -> Graph:
        """Record the library calls `fn` makes on this device into a CUDA graph
        instead of running them.  `fn` must only launch work on buffers that
        already exist (no allocation, download or synchronisation), and one
        uncaptured call of the same shapes must have run before.  The graph's
        `launches` is the number of kernels one replay runs."""
        with self._lock:
            self._require_open()
            before = self.launch_count()
            self._check(self._lib.pb_capture_begin(self._ctx, 0), "pb_capture_begin")
            handle = C.c_void_p()
            try:
                fn()
            except BaseException:
                if self._lib.pb_capture_end(self._ctx, 0, C.byref(handle)) == _lib.PB_OK:
                    self._lib.pb_graph_destroy(self._ctx, 0, handle)
                raise
            self._check(self._lib.pb_capture_end(self._ctx, 0, C.byref(handle)), "pb_capture_end")
            graph = Graph(self, handle.value, self.launch_count() - before)
            self._graphs.add(graph)
            return graph

    # --------------------------------------------------------------- timing
    def launch_count(self) -> int:
        value = C.c_uint64(0)
        self._check(self._lib.pb_launch_count(self._ctx, 0, C.byref(value)), "pb_launch_count")
        return value.value

    def close(self):
        """Free every live buffer and the context (CUDABackend.close,
        src/openpacho/_cuda.py:644-673); arrays become unusable."""
        with self._lock:
            if self._closed:
                return
            self._lib.pb_sync(self._ctx, 0)
            for graph in list(self._graphs):
                graph.close()
            if self._pool is not None:
                self._pool.close()
            for buf in list(self._buffers):
                buf.release()
            self._closed = True
            self._lib.pb_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
