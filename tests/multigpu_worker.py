"""Worker for tests/test_gpu_multi.py: one process per GPU under torchrun.

Checks each sharded path against the oracle on the full (unsharded) input:
the sharded norm (float32 and float64, including a rank with an empty slice)
and the sharded DOT -- both exchanging their partials through the NVLink peer
mailboxes, repeated so both mailbox parities are used -- row-block GEMM with
B broadcast from rank 0, and the batch split of a broadcast-batched GEMM, each
also with its result blocks gathered onto every rank.  With PB_TEST_FAILURE=1
it then has rank 1 leave between steps (nothing in flight) and checks that
rank 0 detects it on the host before launching its next collective and aborts
its communicator.  With PB_TEST_TIMEOUT=1 every rank limits the mailbox wait to
100 ms and rank 0 alone starts a sharded DOT: its merge kernel's wait runs
out, the kernel returns with the error word set (PB_ERR_DEVICE at the next
sync) and the context stays usable.
Each rank writes its results as JSON to ``$PB_RESULT_DIR/rank<r>.json``.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "open-pacho_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main() -> int:
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    out_path = Path(os.environ["PB_RESULT_DIR"]) / f"rank{rank}.json"
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    store = dist.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["PB_STORE_PORT"]), world,
                          rank == 0, timeout=datetime.timedelta(seconds=120))

    import front
    import pacho_b200 as pb
    from oracle import numpy_backend, tolerance
    from pacho_b200 import distributed as D

    be = pb.B200Backend(local)
    group = D.Group(be, rank, world, store, timeout=60)
    res: dict = {"rank": rank}
    # The norm and DOT partials travel through NVLink peer mailboxes.
    res["p2p_unavailable"] = 0 if group.p2p else 1

    for dtype, span in ((np.float32, 35), (np.float64, 300)):
        for n in ((1 << 22) + 5, 1):
            rng = np.random.default_rng(3)
            x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-span, span, n)).astype(dtype)
            s, e = D.shard_range(n, rank, world)
            got = D.sharded_norm(group, front.asarray(x[s:e], backend=be)).item()
            want = numpy_backend.norm(x)
            res[f"norm_{np.dtype(dtype).name}_{n}"] = tolerance.norm_violations(
                np.asarray(got, dtype), np.asarray(want, dtype))

    rng = np.random.default_rng(4)
    n = (1 << 21) + 3
    u = rng.uniform(-1, 1, n).astype(np.float32)
    v = rng.uniform(-1, 1, n).astype(np.float32)
    s, e = D.shard_range(n, rank, world)
    du, dv = front.asarray(u[s:e], backend=be), front.asarray(v[s:e], backend=be)
    for call in range(3):  # three calls: both slot parities, one reused
        d = D.sharded_dot(group, du, dv).item()
        res[f"dot_{call}"] = tolerance.gemm_violations(np.asarray(d, np.float32),
                                                       numpy_backend.dot(u, v), u, v)
    u64, v64 = u.astype(np.float64), v.astype(np.float64)
    d = D.sharded_dot(group, front.asarray(u64[s:e], backend=be), front.asarray(v64[s:e], backend=be)).item()
    res["dot_f64"] = tolerance.gemm_violations(np.asarray(d), numpy_backend.dot(u64, v64), u64, v64)

    for dtype in (np.float32, np.float64):
        A = rng.standard_normal((1000, 300)).astype(dtype)
        B = rng.standard_normal((300, 200)).astype(dtype)
        dB = front.asarray(B if rank == 0 else np.zeros_like(B), backend=be)
        D.broadcast(group, dB, root=0)
        a_local = D.local_rows(A, group)
        c_local = front.asnumpy(D.rowblock_matmul(group, front.asarray(a_local, backend=be), dB))
        res[f"rowblock_{np.dtype(dtype).name}"] = tolerance.gemm_violations(
            c_local, numpy_backend.matmul(a_local, B), a_local, B)

        # The whole C on every rank: row blocks gathered over NCCL (uneven
        # blocks: 1000 rows over 3, 6 or 8 ranks).
        c_all = front.asnumpy(D.rowblock_matmul(group, front.asarray(a_local, backend=be), dB,
                                                gather=True))
        res[f"rowblock_gather_{np.dtype(dtype).name}"] = (
            int(c_all.shape != (1000, 200)) or tolerance.gemm_violations(c_all, numpy_backend.matmul(A, B), A, B))

    A = rng.standard_normal((world + 3, 3, 130, 65)).astype(np.float32)
    B = rng.standard_normal((1, 3, 65, 97)).astype(np.float32)
    a_local = D.local_rows(A, group)
    dA, dB = front.asarray(a_local, backend=be), front.asarray(B, backend=be)
    c_local = front.asnumpy(D.batch_matmul(group, dA, dB))
    res["batch_split"] = tolerance.gemm_violations(c_local, numpy_backend.matmul(a_local, B),
                                                   a_local, B)
    c_all = front.asnumpy(D.batch_matmul(group, dA, dB, gather=True))
    res["batch_split_gather"] = int(c_all.shape != (world + 3, 3, 130, 97)) or tolerance.gemm_violations(
        c_all, numpy_backend.matmul(A, B), A, B)

    be.synchronize()
    if os.environ.get("PB_TEST_TIMEOUT") == "1" and group.p2p:
        # Bounded mailbox wait: every rank limits the wait to 100 ms, rank 0
        # alone starts a sharded DOT (the others never push their partial),
        # and its merge kernel gives up, raises the error word and returns.
        # The context stays usable; the group is out of step and is closed.
        import ctypes as C

        from pacho_b200 import _lib

        lib = be._lib
        _lib.check(lib.pb_peer_set_wait(be._ctx, 0, 100_000_000), "pb_peer_set_wait")
        dist.barrier()
        if rank == 0:
            out = be.empty((1,), np.float32)
            t0 = time.monotonic()
            status = lib.pb_dot_sharded(be._ctx, 0, _lib.PB_F32, e - s, C.c_void_p(du._data.ptr),
                                        C.c_void_p(dv._data.ptr), C.c_void_p(out.ptr))
            sync = lib.pb_sync(be._ctx, 0)
            res["timeout_seconds"] = time.monotonic() - t0
            res["timeout_submit_status"] = status
            res["timeout_sync_status"] = sync
            # The context still works: a local DOT after the expired wait.
            d = front.asnumpy(front.matmul(du, dv))
            res["after_timeout_dot"] = tolerance.gemm_violations(
                np.asarray(d), numpy_backend.dot(u[s:e], v[s:e]), u[s:e], v[s:e])
        dist.barrier()
        group.close()
        dist.barrier()
        dist.destroy_process_group()
        out_path.write_text(json.dumps(res))
        return 0
    if os.environ.get("PB_TEST_FAILURE") == "1":
        dist.barrier()
        if rank == 1:
            group.close()
            res["left"] = True
            out_path.write_text(json.dumps(res))
            return 0
        group.timeout = 5.0
        t0 = time.monotonic()
        try:
            D.sharded_norm(group, front.asarray(np.ones(8, np.float32), backend=be))
            res["failure"] = "not detected"
        except D.RankFailure:
            group.abort()
            res["failure"] = "detected"
        res["failure_seconds"] = time.monotonic() - t0
        out_path.write_text(json.dumps(res))
        return 0
    group.close()
    dist.barrier()
    dist.destroy_process_group()
    out_path.write_text(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
