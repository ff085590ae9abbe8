"""ctypes binding of libpacho_b200.so (declared in include/pacho_b200.h).

The library is located through ``PACHO_B200_LIB`` or next to this file.  A
missing or unloadable library raises :class:`BackendUnavailableError`; there is
no fallback implementation.  Status codes map to exceptions the way the
reference's ``_check`` maps CUDA results (src/openpacho/_cuda.py:49-53).
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

from . import exceptions as _exc

PB_OK = 0
PB_ERR_INVALID = 1
PB_ERR_CUDA = 2
PB_ERR_UNSUPPORTED = 3
PB_ERR_OOM = 4
PB_ERR_NCCL = 5
PB_ERR_DEVICE = 6
PB_ERR_UNAVAILABLE = 7

PB_F32 = 0
PB_F64 = 1
PB_BOOL = 2

PB_GEMM_AUTO = 0
PB_GEMM_SIMT = 1
PB_GEMM_TF32X3 = 2
PB_GEMM_DMMA = 3
PB_GEMM_TF32X3_PRESPLIT = 4
PB_GEMM_TF32X3_FUSED = 5
PB_GEMM_SKINNY = 6

# Elementwise operation codes (pacho_b200.h PB_EW_*), by the reference's
# operation names (src/openpacho/_cuda.py:21-46).
EW_OPS = {name: code for code, name in enumerate((
    "add", "subtract", "multiply", "true_divide", "power", "negative", "positive", "absolute",
    "sqrt", "exp", "log", "sin", "cos", "tanh", "equal", "not_equal", "less", "less_equal",
    "greater", "greater_equal", "isfinite", "cast", "where"))}
EW_OPS["divide"] = EW_OPS["true_divide"]

PB_REDUCE_SUM = 0
PB_REDUCE_MIN = 1
PB_REDUCE_MAX = 2
REDUCE_OPS = {"sum": PB_REDUCE_SUM, "min": PB_REDUCE_MIN, "max": PB_REDUCE_MAX}

LIBRARY_NAME = "libpacho_b200.so"

_i = C.c_int
_i64 = C.c_int64
_sz = C.c_size_t
_p = C.c_void_p
_pi64 = C.POINTER(C.c_int64)
_ctx = C.c_void_p

# name -> (argtypes); every function returns int except pb_last_error.
PROTOTYPES = {
    "pb_abi_version": [],
    "pb_device_count": [C.POINTER(C.c_int)],
    "pb_driver_version": [C.POINTER(C.c_int)],
    "pb_device_info": [_i, C.c_char_p, _sz, C.POINTER(C.c_size_t), C.POINTER(C.c_int),
                       C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "pb_init": [_i, C.POINTER(C.c_int), C.POINTER(_ctx)],
    "pb_destroy": [_ctx],
    "pb_alloc": [_ctx, _i, _sz, C.POINTER(_p)],
    "pb_free": [_ctx, _i, _p],
    "pb_h2d": [_ctx, _i, _p, _p, _sz, _i],
    "pb_d2h": [_ctx, _i, _p, _p, _sz],
    "pb_d2h_async": [_ctx, _i, _p, _p, _sz],
    "pb_d2d": [_ctx, _i, _p, _p, _sz],
    "pb_fill": [_ctx, _i, _i, _p, _sz, C.c_double],
    "pb_sync": [_ctx, _i],
    "pb_host_register": [_p, _sz],
    "pb_host_unregister": [_p],
    "pb_trim": [_ctx, _i],
    "pb_timer_start": [_ctx, _i],
    "pb_timer_stop": [_ctx, _i, C.POINTER(C.c_float)],
    "pb_launch_count": [_ctx, _i, C.POINTER(C.c_uint64)],
    "pb_ktimer_enable": [_ctx, _i, _i],
    "pb_ktimer_read": [_ctx, _i, C.POINTER(C.c_double), C.POINTER(C.c_uint64)],
    "pb_memory_stats": [_ctx, _i, C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz)],
    "pb_peer_enable": [_ctx, C.POINTER(C.c_int)],
    "pb_alloc_mapped": [_ctx, _i, _sz, C.POINTER(C.c_void_p)],
    "pb_free_mapped": [_ctx, _i, C.c_void_p],
    "pb_copy_peer": [_ctx, _i, C.c_void_p, _i, C.c_void_p, _sz, _i, _i],
    "pb_stream_wait": [_ctx, _i, _i, _i, _i],
    "pb_capture_begin": [_ctx, _i],
    "pb_capture_end": [_ctx, _i, C.POINTER(C.c_void_p)],
    "pb_graph_launch": [_ctx, _i, C.c_void_p],
    "pb_graph_destroy": [_ctx, _i, C.c_void_p],
    "pb_gemm": [_ctx, _i, _i, _i, _pi64, _pi64, _pi64, _i64, _i64, _i64, _p, _p, _p],
    "pb_gemm_ex": [_ctx, _i, _i, _i, _pi64, _pi64, _pi64, _i64, _i64, _i64, _p, _p, _p, _i],
    "pb_gemm_host": [_ctx, _i, _i, _i, _pi64, _pi64, _pi64, _i64, _i64, _i64, _p, _p, _p, _i],
    "pb_gemv": [_ctx, _i, _i, _i64, _i64, _p, _p, _p],
    "pb_gemv_residual": [_ctx, _i, _i, _i64, _i64, _p, _p, _p, _p],
    "pb_elementwise": [_ctx, _i, _i, _i, C.POINTER(_p), C.POINTER(_i), _pi64, _i, _pi64, _i, _p],
    "pb_gather": [_ctx, _i, _i, _p, _i, _pi64, _i64, _pi64, _p],
    "pb_reduce": [_ctx, _i, _i, _i, _p, _i, _pi64, C.c_uint32, _i, _p],
    "pb_dot": [_ctx, _i, _i, _i64, _p, _p, _p],
    "pb_dot_noalloc": [_ctx, _i, _i, _i64, _p, _p, _p],
    "pb_peer_export": [_ctx, _i, _i, _i, C.c_char_p],
    "pb_peer_import": [_ctx, _i, _i, C.c_char_p],
    "pb_peer_close": [_ctx, _i],
    "pb_peer_set_wait": [_ctx, _i, C.c_uint64],
    "pb_dot_sharded": [_ctx, _i, _i, _i64, _p, _p, _p],
    "pb_norm": [_ctx, _i, _i, _i64, _i64, _i64, _p, _p],
    "pb_norm_strided": [_ctx, _i, _i, _i, _pi64, _pi64, _i, _pi64, _pi64, _p, _p],
    "pb_comm_unique_id": [C.c_char_p],
    "pb_comm_init": [_ctx, _i, _i, _i, C.c_char_p],
    "pb_comm_destroy": [_ctx, _i],
    "pb_comm_abort": [_ctx, _i],
    "pb_broadcast": [_ctx, _i, _p, _sz, _i],
    "pb_norm_sharded": [_ctx, _i, _i, _i64, _p, _p],
    "pb_allreduce_sum": [_ctx, _i, _i, _p, _sz],
}


class B200Error(RuntimeError):
    """A libpacho_b200 call failed after the backend was initialised."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    override = os.environ.get("PACHO_B200_LIB")
    return Path(override) if override else Path(__file__).resolve().parent / LIBRARY_NAME


def load():
    """Load and type the shared library once; raise if it is unavailable."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise _exc.BackendUnavailableError(
                f"{LIBRARY_NAME} not found at {path}; build it with "
                "`python -m pacho_b200._build` (nvcc, sm_100a)"
            )
        try:
            lib = C.CDLL(str(path))
        except OSError as exc:
            raise _exc.BackendUnavailableError(f"cannot load {path}: {exc}") from exc
        lib.pb_last_error.restype = C.c_char_p
        lib.pb_last_error.argtypes = []
        for name, args in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = C.c_int
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().pb_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(status: int, what: str = "b200 call") -> None:
    """Raise the exception that matches a non-zero status."""
    if status == PB_OK:
        return
    message = f"{what} failed: {last_error()}"
    if status == PB_ERR_UNAVAILABLE:
        raise _exc.BackendUnavailableError(message)
    if status == PB_ERR_INVALID:
        raise ValueError(message)
    if status == PB_ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    if status == PB_ERR_OOM:
        raise MemoryError(message)
    raise B200Error(status, message)


def dtype_code(dtype) -> int:
    import numpy as np

    dtype = np.dtype(dtype)
    if dtype == np.float32:
        return PB_F32
    if dtype == np.float64:
        return PB_F64
    if dtype == np.bool_:
        return PB_BOOL
    raise _exc.UnsupportedDtypeError(f"b200 backend supports bool, float32 and float64, not {dtype}")


def i64_array(values):
    values = list(values)
    return (C.c_int64 * max(1, len(values)))(*values)
