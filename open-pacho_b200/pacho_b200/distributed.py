"""Multi-GPU use of the b200 backend: one process per GPU, NCCL over NVLink.

OpenPacho is single-device (src/openpacho/_cuda.py:138-199); this module adds
the sharded forms of its hot path that split naturally:

* :func:`shard_range` -- balanced contiguous partition (rows, batches, slices);
* :class:`Group` -- a communicator of ``world`` processes: the NCCL unique id
  travels through any key-value store with ``set``/``get`` (for example
  ``torch.distributed.TCPStore``); a per-step heartbeat lets ranks detect a
  departed peer on the host *before* launching a collective;
* :func:`sharded_norm` -- global Euclidean norm of a vector sliced across ranks
  (local (scale, ssq) pairs exchanged and merged in rank order);
* :func:`sharded_dot` -- global DOT of sliced vectors (local DOT + sum);
* :func:`rowblock_matmul` -- row blocks of A per rank, B broadcast from a root;
* :func:`batch_matmul` -- the leading batch dimension split across ranks.

No data-path collective is used where the work is independent (row blocks,
batch split); the broadcast of B happens once per operand.  The norm and DOT
partials travel through peer mailboxes (CUDA IPC mappings of each rank's
small slot array, set up when the group forms): NVLink stores from the
kernels and a bounded wait, with NCCL as the fallback where IPC is not
available (``Group.p2p`` says which; ``PB_P2P=0`` forces NCCL).
"""

from __future__ import annotations

import ctypes as C
import os
import time

import numpy as np

from . import _lib
from .api import asarray, ndarray
from .backend import B200Backend


class RankFailure(RuntimeError):
    """A peer did not reach a step in time; no collective was launched."""


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n`` items for ``rank`` of ``world``; the
    first ``n % world`` ranks take one extra item."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} rank={rank} world={world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _store_get(store, key: str, timeout: float) -> bytes:
    deadline = time.monotonic() + timeout
    while True:
        try:
            if hasattr(store, "check") and not store.check([key]):
                raise KeyError(key)
            return bytes(store.get(key))
        except Exception:  # noqa: BLE001 - store-specific "missing" errors
            if time.monotonic() > deadline:
                raise RankFailure(f"timed out after {timeout:.1f}s waiting for {key!r}") from None
            time.sleep(0.01)


class Group:
    """NCCL communicator for one GPU per process.

    ``store`` needs ``set(key, value)`` and ``get(key)`` (and optionally
    ``check(keys)``); ``prefix`` separates several groups on one store."""

    def __init__(self, backend: B200Backend, rank: int, world: int, store, *, prefix: str = "pb",
                 timeout: float = 60.0):
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"bad rank {rank} of {world}")
        self.backend, self.rank, self.world = backend, rank, world
        self.store, self.prefix, self.timeout = store, prefix, timeout
        self._step = 0
        self._joined = False
        self.p2p = False
        lib = backend._lib
        if world == 1:
            return
        if rank == 0:
            uid = C.create_string_buffer(128)
            _lib.check(lib.pb_comm_unique_id(uid), "pb_comm_unique_id")
            store.set(f"{prefix}/nccl_id", uid.raw)
            raw = uid.raw
        else:
            raw = _store_get(store, f"{prefix}/nccl_id", timeout)
        if len(raw) != 128:
            raise RuntimeError("malformed NCCL unique id from the store")
        with backend._lock:
            _lib.check(lib.pb_comm_init(backend._ctx, 0, world, rank, raw), "pb_comm_init")
        self._joined = True
        if os.environ.get("PB_P2P", "1") != "0" and world <= 8:
            self.p2p = self._map_mailboxes()

    def _map_mailboxes(self) -> bool:
        """Export this rank's mailbox, map every peer's; every rank agrees
        on the outcome through the store, so all use the same path."""
        lib, b, key = self.backend._lib, self.backend, f"{self.prefix}/box"
        handle = C.create_string_buffer(64)
        with b._lock:
            ok = lib.pb_peer_export(b._ctx, 0, self.world, self.rank, handle) == _lib.PB_OK
        self.store.set(f"{key}/{self.rank}", handle.raw if ok else b"")
        handles = [_store_get(self.store, f"{key}/{r}", self.timeout) for r in range(self.world)]
        ok = ok and all(len(h) == 64 for h in handles)
        if ok:
            with b._lock:
                ok = lib.pb_peer_import(b._ctx, 0, self.world, b"".join(handles)) == _lib.PB_OK
        self.store.set(f"{key}/ok/{self.rank}", b"1" if ok else b"0")
        agreed = all(_store_get(self.store, f"{key}/ok/{r}", self.timeout) == b"1"
                     for r in range(self.world))
        if not agreed:
            with b._lock:
                lib.pb_peer_close(b._ctx, 0)
        return agreed

    def heartbeat(self):
        """Announce this rank at the next step and wait (bounded) for every
        peer; raises RankFailure, before any collective, if one is missing."""
        if self.world == 1:
            return
        step = self._step
        self._step += 1
        self.store.set(f"{self.prefix}/alive/{step}/{self.rank}", b"1")
        for r in range(self.world):
            if r != self.rank:
                _store_get(self.store, f"{self.prefix}/alive/{step}/{r}", self.timeout)

    def close(self):
        if self._joined:
            with self.backend._lock:
                self.backend._lib.pb_peer_close(self.backend._ctx, 0)
                self.backend._lib.pb_comm_destroy(self.backend._ctx, 0)
            self._joined = False

    def abort(self):
        """Drop the communicator without waiting for peers (after RankFailure)."""
        if self._joined:
            with self.backend._lock:
                self.backend._lib.pb_peer_close(self.backend._ctx, 0)
                self.backend._lib.pb_comm_abort(self.backend._ctx, 0)
            self._joined = False

    def __enter__(self):
        return self

    def __exit__(self, exc_type, *exc):
        if exc_type is RankFailure:
            self.abort()
        else:
            self.close()


def _buf(a: ndarray) -> C.c_void_p:
    return C.c_void_p(a._data.ptr)


def sharded_norm(group: Group, x_local: ndarray) -> ndarray:
    """Euclidean norm of the concatenation of every rank's ``x_local``
    (any shape, flattened; may be empty).  Every rank gets the result."""
    b = group.backend
    dtype = b.validate_dtype(x_local.dtype)
    out = b.empty((1,), dtype)
    if group.world == 1:
        n = x_local.size
        with b._lock:
            if n:
                _lib.check(b._lib.pb_norm(b._ctx, 0, _lib.dtype_code(dtype), 1, n, 1, _buf(x_local),
                                          C.c_void_p(out.ptr)), "pb_norm")
            else:
                _lib.check(b._lib.pb_fill(b._ctx, 0, _lib.dtype_code(dtype), C.c_void_p(out.ptr), 1,
                                          0.0), "pb_fill")
        return ndarray._wrap(out, (), dtype, b)
    group.heartbeat()
    with b._lock:
        _lib.check(b._lib.pb_norm_sharded(b._ctx, 0, _lib.dtype_code(dtype), x_local.size,
                                          _buf(x_local) if x_local.size else None, C.c_void_p(out.ptr)),
                   "pb_norm_sharded")
    return ndarray._wrap(out, (), dtype, b)


def sharded_dot(group: Group, u_local: ndarray, v_local: ndarray) -> ndarray:
    """DOT of vectors sliced identically across ranks; every rank gets it."""
    b = group.backend
    if u_local.shape != v_local.shape or u_local.ndim != 1:
        raise ValueError("sharded_dot takes equal 1-D slices")
    dtype = b.validate_dtype(np.result_type(u_local.dtype, v_local.dtype))
    out = b.empty((1,), dtype)
    code = _lib.dtype_code(dtype)
    if group.p2p:
        group.heartbeat()
        with b._lock:
            _lib.check(b._lib.pb_dot_sharded(b._ctx, 0, code, u_local.size, _buf(u_local),
                                             _buf(v_local), C.c_void_p(out.ptr)), "pb_dot_sharded")
        return ndarray._wrap(out, (), dtype, b)
    with b._lock:
        _lib.check(b._lib.pb_dot(b._ctx, 0, code, u_local.size, _buf(u_local), _buf(v_local),
                                 C.c_void_p(out.ptr)), "pb_dot")
    if group.world > 1:
        group.heartbeat()
        with b._lock:
            _lib.check(b._lib.pb_allreduce_sum(b._ctx, 0, code, C.c_void_p(out.ptr), 1),
                       "pb_allreduce_sum")
    return ndarray._wrap(out, (), dtype, b)


def broadcast(group: Group, a: ndarray, root: int = 0) -> ndarray:
    """In-place broadcast of ``a`` (same shape and dtype on every rank)."""
    if group.world > 1:
        b = group.backend
        group.heartbeat()
        with b._lock:
            _lib.check(b._lib.pb_broadcast(b._ctx, 0, _buf(a), a.nbytes, root), "pb_broadcast")
    return a


def rowblock_matmul(group: Group, a_local: ndarray, b: ndarray) -> ndarray:
    """``a_local @ b`` where ``a_local`` is this rank's row block of A and
    ``b`` is already on every rank (see :func:`broadcast`).  Returns this
    rank's row block of C; no collective on the data path."""
    from .api import matmul

    return matmul(a_local, b)


def batch_matmul(group: Group, a_local: ndarray, b: ndarray) -> ndarray:
    """Batched ``a_local @ b`` for this rank's slice of the leading batch
    dimension of A (B broadcasts over it)."""
    from .api import matmul

    return matmul(a_local, b)


def local_rows(a: np.ndarray, group: Group) -> np.ndarray:
    """This rank's contiguous block of rows (axis 0) of a host array."""
    start, stop = shard_range(a.shape[0], group.rank, group.world)
    return np.ascontiguousarray(a[start:stop])


def upload_local(a: np.ndarray, group: Group) -> ndarray:
    return asarray(local_rows(a, group), backend=group.backend)


__all__ = [
    "Group",
    "RankFailure",
    "batch_matmul",
    "broadcast",
    "local_rows",
    "rowblock_matmul",
    "shard_range",
    "sharded_dot",
    "sharded_norm",
    "upload_local",
]

