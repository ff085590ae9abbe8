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
* :func:`rowblock_matmul` -- row blocks of A per rank, B broadcast from a root,
  optionally the row blocks of C gathered onto every rank;
* :func:`batch_matmul` -- the leading batch dimension split across ranks
  (B broadcasting over it), optionally gathered;
* :func:`scatter_rows` / :func:`gather_rows` -- this rank's block of a host
  array on its GPU, and the blocks of every rank assembled on every GPU
  (one NCCL broadcast per rank into its rows, uneven blocks allowed).

Arrays are anything with the backend protocol's ``shape``/``dtype``/``_data``
(OpenPacho arrays on the b200 backend, or :class:`~pacho_b200.backend.DeviceArray`);
results come back as the same kind.

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
from .backend import B200Backend, DeviceArray, wrap_like


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

    def exchange(self, tag: str, value: int) -> list[int]:
        """Every rank's integer ``value`` for ``tag``, in rank order (host store)."""
        if self.world == 1:
            return [int(value)]
        key = f"{self.prefix}/x/{tag}"
        self.store.set(f"{key}/{self.rank}", str(int(value)).encode())
        return [int(_store_get(self.store, f"{key}/{r}", self.timeout)) for r in range(self.world)]

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


def _buf(a) -> C.c_void_p:
    return C.c_void_p(a._data.ptr)


def _scalar(template, out, dtype, backend):
    return wrap_like(template, out, (), dtype, backend)


def sharded_norm(group: Group, x_local):
    """Euclidean norm of the concatenation of every rank's ``x_local``
    (any shape, flattened; may be empty).  Every rank gets the result."""
    b = group.backend
    dtype = b.validate_dtype(x_local.dtype)
    out = b.empty((1,), dtype)
    n = int(np.prod(x_local.shape))
    if group.world == 1:
        with b._lock:
            if n:
                _lib.check(b._lib.pb_norm(b._ctx, 0, _lib.dtype_code(dtype), 1, n, 1, _buf(x_local),
                                          C.c_void_p(out.ptr)), "pb_norm")
            else:
                _lib.check(b._lib.pb_fill(b._ctx, 0, _lib.dtype_code(dtype), C.c_void_p(out.ptr), 1,
                                          0.0), "pb_fill")
        return _scalar(x_local, out, dtype, b)
    group.heartbeat()
    with b._lock:
        _lib.check(b._lib.pb_norm_sharded(b._ctx, 0, _lib.dtype_code(dtype), n,
                                          _buf(x_local) if n else None, C.c_void_p(out.ptr)),
                   "pb_norm_sharded")
    return _scalar(x_local, out, dtype, b)


def sharded_dot(group: Group, u_local, v_local):
    """DOT of vectors sliced identically across ranks; every rank gets it."""
    b = group.backend
    if tuple(u_local.shape) != tuple(v_local.shape) or len(u_local.shape) != 1:
        raise ValueError("sharded_dot takes equal 1-D slices")
    dtype = b.validate_dtype(np.result_type(u_local.dtype, v_local.dtype))
    if u_local.dtype != dtype or v_local.dtype != dtype:
        raise NotImplementedError("sharded_dot needs both slices in the result dtype")
    out = b.empty((1,), dtype)
    code = _lib.dtype_code(dtype)
    n = u_local.shape[0]
    if group.p2p:
        group.heartbeat()
        with b._lock:
            _lib.check(b._lib.pb_dot_sharded(b._ctx, 0, code, n, _buf(u_local), _buf(v_local),
                                             C.c_void_p(out.ptr)), "pb_dot_sharded")
        return _scalar(u_local, out, dtype, b)
    with b._lock:
        _lib.check(b._lib.pb_dot(b._ctx, 0, code, n, _buf(u_local), _buf(v_local),
                                 C.c_void_p(out.ptr)), "pb_dot")
    if group.world > 1:
        group.heartbeat()
        with b._lock:
            _lib.check(b._lib.pb_allreduce_sum(b._ctx, 0, code, C.c_void_p(out.ptr), 1),
                       "pb_allreduce_sum")
    return _scalar(u_local, out, dtype, b)


def broadcast(group: Group, a, root: int = 0):
    """In-place broadcast of ``a`` (same shape and dtype on every rank)."""
    if group.world > 1:
        b = group.backend
        nbytes = int(np.prod(a.shape)) * np.dtype(a.dtype).itemsize
        group.heartbeat()
        with b._lock:
            _lib.check(b._lib.pb_broadcast(b._ctx, 0, _buf(a), nbytes, root), "pb_broadcast")
    return a


def _matmul(group: Group, a, b):
    """``a @ b`` on this rank's GPU through the backend protocol."""
    be = group.backend
    dtype = be.validate_dtype(np.result_type(a.dtype, b.dtype))
    if a.dtype != dtype or b.dtype != dtype:
        raise NotImplementedError("sharded matmul needs both operands in the result dtype")
    if len(a.shape) < 2 or len(b.shape) < 2:
        raise ValueError("sharded matmul takes matrices (or batches of them)")
    if a.shape[-1] != b.shape[-2]:
        raise ValueError("matmul inner dimensions do not match")
    batch = np.broadcast_shapes(tuple(a.shape[:-2]), tuple(b.shape[:-2]))
    shape = tuple(batch) + (a.shape[-2], b.shape[-1])
    return wrap_like(a, be.matmul(a, b, shape, dtype), shape, dtype, be)


def gather_rows(group: Group, local):
    """Every rank's block of rows (leading dimension; the trailing
    dimensions equal on all ranks) stacked in rank order, on every rank.  One
    NCCL broadcast per rank, in place into that rank's rows of the result;
    the blocks may differ in length."""
    be = group.backend
    if group.world == 1:
        return local
    rows = group.exchange(f"gather/{group._step}", local.shape[0] if local.shape else 0)
    trailing = tuple(local.shape[1:])
    row_bytes = int(np.prod(trailing)) * np.dtype(local.dtype).itemsize
    shape = (sum(rows),) + trailing
    out = be.empty(shape, local.dtype)
    offsets = np.concatenate([[0], np.cumsum(rows)]).astype(int)
    mine = rows[group.rank] * row_bytes
    with be._lock:
        if mine:
            _lib.check(be._lib.pb_d2d(be._ctx, 0, C.c_void_p(out.ptr + int(offsets[group.rank]) * row_bytes),
                                      _buf(local), mine), "pb_d2d")
    group.heartbeat()
    with be._lock:
        for r in range(group.world):
            if rows[r]:
                _lib.check(be._lib.pb_broadcast(be._ctx, 0, C.c_void_p(out.ptr + int(offsets[r]) * row_bytes),
                                                rows[r] * row_bytes, r), "pb_broadcast")
    return wrap_like(local, out, shape, local.dtype, be)


def rowblock_matmul(group: Group, a_local, b, *, gather: bool = False):
    """``a_local @ b`` where ``a_local`` is this rank's row block of A and
    ``b`` is on every rank (see :func:`broadcast`): this rank's row block of C,
    with no collective on the data path; ``gather=True`` returns the whole C
    on every rank (:func:`gather_rows`)."""
    c_local = _matmul(group, a_local, b)
    return gather_rows(group, c_local) if gather else c_local


def batch_matmul(group: Group, a_local, b, *, gather: bool = False):
    """Batched ``a_local @ b`` for this rank's slice of the leading batch
    dimension of A, B broadcasting over it; with
    ``gather=True`` every rank gets the whole batched product."""
    if len(a_local.shape) < 3:
        raise ValueError("batch_matmul splits a leading batch dimension of A")
    c_local = _matmul(group, a_local, b)
    return gather_rows(group, c_local) if gather else c_local


def local_rows(a: np.ndarray, group: Group) -> np.ndarray:
    """This rank's contiguous block of rows (axis 0) of a host array."""
    start, stop = shard_range(a.shape[0], group.rank, group.world)
    return np.ascontiguousarray(a[start:stop])


def scatter_rows(a: np.ndarray, group: Group) -> DeviceArray:
    """This rank's row block of host array ``a`` (every rank holds ``a``) on
    its GPU."""
    block = local_rows(a, group)
    return DeviceArray(group.backend, group.backend.upload(block), block.shape, block.dtype)


upload_local = scatter_rows


__all__ = [
    "Group",
    "RankFailure",
    "batch_matmul",
    "broadcast",
    "gather_rows",
    "local_rows",
    "rowblock_matmul",
    "scatter_rows",
    "shard_range",
    "sharded_dot",
    "sharded_norm",
    "upload_local",
]

