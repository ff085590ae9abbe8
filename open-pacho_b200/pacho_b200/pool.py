"""Several GPUs behind one backend object, in one process.

``set_backend("b200", device="0-7")`` (OpenPacho's selection call,
src/openpacho/backends.py:217-231) gives a :class:`~pacho_b200.B200Backend`
whose context holds every listed GPU.  Arrays live on the first one (the
primary).  A matrix product large enough to pay for the NVLink transfers is
split into row blocks (or blocks of its leading batch dimension) across all
of them: each other GPU receives its block of A and the whole of B by peer
copies, computes its block of C, and copies it back into the result on the
primary.  B travels as a chain (primary -> 1 -> 2 -> ...) cut into chunks, so
every link carries it once and the hops overlap.  Memory-bound operations
(GEMV, DOT, norms, elementwise) stay on the primary: moving an operand over
NVLink costs more than reading it once from the primary's own HBM.

The reference drives one device per backend object
(src/openpacho/_cuda.py:138-199); this is the B200 addition its
``device=`` argument has room for.
"""

from __future__ import annotations

import ctypes as C
import re
from dataclasses import dataclass
from math import prod

from . import _lib

# Rates the split decision assumes for one GPU (TFLOP/s sustained, 3xTF32 /
# DMMA) and for the primary's NVLink traffic (bytes/s per direction).
GEMM_RATE = {4: 180e12, 8: 30e12}
LINK_BYTES_PER_S = 700e9
# Split only when the estimate is at most this fraction of one GPU's time.
MIN_GAIN = 0.7
CHUNK_BYTES = 64 << 20
ROW_ALIGN = 128  # the GEMM tile height


def parse_devices(device=None, gpus=None) -> list[int]:
    """CUDA ordinals from OpenPacho's ``device=`` value: ``None`` or an int
    or ``"3"`` (one GPU), ``"0-7"`` (a range), ``"0,2,5"`` (a list), each
    optionally prefixed ``"cuda:"``; ``gpus=N`` takes N consecutive ordinals
    from the first one given."""
    if device is None:
        ordinals = [0]
    elif isinstance(device, int):
        ordinals = [device]
    else:
        text = str(device).strip()
        if text.lower().startswith("cuda:"):
            text = text[5:]
        ordinals = []
        for part in text.split(","):
            part = part.strip()
            m = re.fullmatch(r"(\d+)\s*-\s*(\d+)", part)
            if m:
                lo, hi = int(m.group(1)), int(m.group(2))
                if hi < lo:
                    raise ValueError(f"empty device range {part!r}")
                ordinals.extend(range(lo, hi + 1))
            elif part.isdigit():
                ordinals.append(int(part))
            else:
                raise ValueError(f"b200 device must be an ordinal, a range or a list, not {device!r}")
    if gpus is not None:
        gpus = int(gpus)
        if gpus < 1:
            raise ValueError("gpus must be at least 1")
        if len(ordinals) == 1:
            ordinals = list(range(ordinals[0], ordinals[0] + gpus))
        elif gpus != len(ordinals):
            raise ValueError(f"gpus={gpus} does not match device={device!r}")
    if len(set(ordinals)) != len(ordinals):
        raise ValueError(f"b200 device list repeats an ordinal: {device!r}")
    return ordinals


def blocks(total: int, parts: int, align: int = 1) -> list[tuple[int, int]]:
    """Split range(total) into `parts` contiguous blocks, boundaries on
    multiples of `align` where possible, sizes as equal as that allows;
    empty blocks are dropped."""
    units = -(-total // align)
    base, extra = divmod(units, parts)
    out, start = [], 0
    for p in range(parts):
        stop = min(total, start + (base + (p < extra)) * align)
        if stop > start:
            out.append((start, stop))
        start = stop
    return out


@dataclass(frozen=True)
class Split:
    """How one product is cut: `outer` leading blocks (batch entries or
    rows), each block `a_block`/`c_block` elements of A and C; B is sliced
    along the same blocks when `b_block` is nonzero, else copied whole."""

    outer: int
    a_block: int
    b_block: int
    c_block: int
    b_whole: int
    m: int
    n: int
    k: int
    batch: tuple


def plan(a_shape, b_shape, batch, m, n, k) -> Split | None:
    """The cut for ``a @ b`` with broadcast batch `batch`, or None when the
    layout has no contiguous blocks (A broadcast along the leading batch
    dimension, or a partially broadcast B)."""
    a_batch = tuple(a_shape[:-2])
    b_batch = tuple(b_shape[:-2])
    if not batch:
        return Split(m, k, 0, n, k * n, m, n, k, ())
    if a_batch != tuple(batch):
        return None
    inner = prod(batch[1:])
    if b_batch == tuple(batch):
        return Split(batch[0], inner * m * k, inner * k * n, inner * m * n, 0, m, n, k, tuple(batch))
    if not b_batch:
        return Split(batch[0], inner * m * k, 0, inner * m * n, k * n, m, n, k, tuple(batch))
    return None


def worth_splitting(flops: float, itemsize: int, a_bytes: int, b_bytes: int, c_bytes: int,
                    ndev: int, rate: float | None = None, min_gain: float = MIN_GAIN) -> bool:
    """Whether `ndev` GPUs beat one: compute shrinks by ndev, the primary
    sends the other blocks of A and B once and receives the other blocks of
    C (its busiest link bounds the transfers)."""
    if ndev < 2:
        return False
    rate = rate or GEMM_RATE.get(itemsize, 30e12)
    one = flops / rate
    moved = (a_bytes + c_bytes) * (ndev - 1) / ndev + b_bytes
    split = one / ndev + moved / LINK_BYTES_PER_S
    return split <= min_gain * one


class DevicePool:
    """The GEMM split over a backend's devices (indices 0..ndev-1 of its
    context, 0 = primary).

    Peer access maps cudaMalloc memory into the other devices but not the
    stream-ordered pools the arrays live in, so every copy is issued by the
    device that owns the pool side of it and reaches the other side through
    a mapped workspace: the primary pushes the blocks of A into each
    device's workspace and pulls the blocks of C back out of them; B goes
    down the chain, each device pushing each chunk on to the next.  The
    workspaces (A, B and C per device) are grow-only and kept between calls.
    """

    def __init__(self, backend, ndev: int):
        self.b, self.ndev = backend, ndev
        self.lib, self.ctx = backend._lib, backend._ctx
        flag = C.c_int(0)
        _lib.check(self.lib.pb_peer_enable(self.ctx, C.byref(flag)), "pb_peer_enable")
        self.all_peer = bool(flag.value)
        self.splits = 0  # products run split (for tests and the bench)
        self.ws = {}  # (device, role) -> (pointer, bytes)

    def _workspace(self, dev, role, nbytes):
        ptr, have = self.ws.get((dev, role), (0, 0))
        if have >= nbytes:
            return ptr
        if ptr:
            # Copies on other devices' streams may still read it.
            for i in range(self.ndev):
                _lib.check(self.lib.pb_sync(self.ctx, i), "pb_sync")
            _lib.check(self.lib.pb_free_mapped(self.ctx, dev, C.c_void_p(ptr)), "pb_free_mapped")
            del self.ws[(dev, role)]
        out = C.c_void_p()
        _lib.check(self.lib.pb_alloc_mapped(self.ctx, dev, max(int(nbytes), 1), C.byref(out)),
                   "pb_alloc_mapped")
        self.ws[(dev, role)] = (out.value, int(nbytes))
        return out.value

    def close(self):
        """Frees the workspaces (after the primary's stream, which ends
        after every device's work)."""
        self.lib.pb_sync(self.ctx, 0)
        for (dev, _), (ptr, _) in list(self.ws.items()):
            self.lib.pb_free_mapped(self.ctx, dev, C.c_void_p(ptr))
        self.ws.clear()

    def matmul(self, code, itemsize, sp: Split, A: int, B: int, O: int, gemm) -> None:
        """C = A @ B by blocks of `sp.outer`; `gemm(dev, outer, A, B, C)`
        launches one block's product on device index `dev`.  Called with the
        backend's lock held; the primary's stream ends after every block.

        Each device has its kernel stream (0) and a copy stream (1).  The
        primary pushes and pulls on its copy stream, so its own block starts
        at once and each other block's result is pulled as soon as it is
        done; the chain hops of B run on the copy streams of the devices
        that forward them."""
        lib, ctx = self.lib, self.ctx
        check = _lib.check
        align = ROW_ALIGN if not sp.batch else 1
        parts = blocks(sp.outer, self.ndev, align)
        n = len(parts)
        placed = [(A, B, O)]
        for d, (lo, hi) in enumerate(parts[1:], start=1):
            rows = hi - lo
            a = self._workspace(d, "a", rows * sp.a_block * itemsize)
            b = self._workspace(d, "b", (sp.b_block * rows if sp.b_block else sp.b_whole) * itemsize)
            c = self._workspace(d, "c", rows * sp.c_block * itemsize)
            placed.append((a, b, c))

        def wait(w, ws, g, gs):
            check(lib.pb_stream_wait(ctx, w, ws, g, gs), "pb_stream_wait")

        def copy(dst_dev, dst, src_dev, src, nbytes, on):
            check(lib.pb_copy_peer(ctx, dst_dev, C.c_void_p(dst), src_dev, C.c_void_p(src), nbytes, on, 1),
                  "pb_copy_peer")

        try:
            # Every stream starts after the primary's kernel stream, whose
            # last call ended after every device's work: inputs are ready
            # and the workspaces free.
            wait(0, 1, 0, 0)
            for d in range(1, n):
                wait(d, 0, 0, 0)
                wait(d, 1, 0, 0)
            # The primary pushes the blocks of A (and of a batched B).
            for d, (lo, hi) in enumerate(parts[1:], start=1):
                rows = hi - lo
                copy(d, placed[d][0], 0, A + lo * sp.a_block * itemsize, rows * sp.a_block * itemsize, 0)
                if sp.b_block:
                    copy(d, placed[d][1], 0, B + lo * sp.b_block * itemsize, rows * sp.b_block * itemsize, 0)
            if not sp.b_block and n > 1:
                # The whole B down the chain, chunk by chunk: device d - 1
                # forwards a chunk once its own copy of it has landed.
                total = sp.b_whole * itemsize
                for off in range(0, total, CHUNK_BYTES):
                    size = min(CHUNK_BYTES, total - off)
                    for d in range(1, n):
                        if d > 1:
                            wait(d - 1, 1, d - 2, 1)
                        copy(d, placed[d][1] + off, d - 1, placed[d - 1][1] + off, size, d - 1)
            # Each device's block after the pushes into it (all joins queued
            # before any block, so no device waits for another's product).
            for d in range(1, n):
                wait(d, 0, 0, 1)
                if d > 1 and not sp.b_block:
                    wait(d, 0, d - 1, 1)
            for d in range(1, n):
                lo, hi = parts[d]
                gemm(d, hi - lo, *placed[d])
            gemm(0, parts[0][1] - parts[0][0], A, B, O)
            # The primary pulls each block of C as it is done.
            for d, (lo, hi) in enumerate(parts[1:], start=1):
                wait(0, 1, d, 0)
                copy(0, O + lo * sp.c_block * itemsize, d, placed[d][2], (hi - lo) * sp.c_block * itemsize, 0)
            self.splits += 1
        finally:
            # Whatever happened, the primary's kernel stream ends after its
            # copy stream and every device's work (so the result is complete
            # there and the workspaces are free for the next call).
            lib.pb_stream_wait(ctx, 0, 0, 0, 1)
            for d in range(1, n):
                lib.pb_stream_wait(ctx, 0, 0, d, 0)
                lib.pb_stream_wait(ctx, 0, 0, d, 1)
