"""Host-side logic of the multi-GPU layer, as two or four gloo ranks on CPU.

Covers the partitioning, the NCCL-id rendezvous through a TCP store and the
heartbeat that detects a departed rank before any collective is launched.
The communicator calls go to a recording fake (no GPU here); the GPU path
itself is exercised by tests/test_gpu_multi.py on 2 GPUs.
"""

from __future__ import annotations

import ctypes as C
import datetime
import multiprocessing as mp
import os
import socket
import threading
import time

import pytest

from pacho_b200.distributed import Group, RankFailure, shard_range

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeCommLib:
    def __init__(self, all_export=False):
        self.calls = []
        self.all_export = all_export

    def pb_comm_unique_id(self, buf):
        C.memmove(buf, bytes(range(128)), 128)
        self.calls.append(("uid",))
        return 0

    def pb_comm_init(self, ctx, dev, world, rank, raw):
        self.calls.append(("init", world, rank, bytes(raw)))
        return 0

    def pb_comm_destroy(self, ctx, dev):
        self.calls.append(("destroy",))
        return 0

    def pb_comm_abort(self, ctx, dev):
        self.calls.append(("abort",))
        return 0

    def pb_peer_export(self, ctx, dev, world, rank, handle):
        # Rank 0 can export, rank 1 cannot (no CUDA IPC): every rank must then
        # agree on the NCCL path and rank 0 must unmap what it set up.
        # With all_export every rank exports a handle of 64 bytes of its rank.
        self.calls.append(("export", rank))
        if rank == 0 or self.all_export:
            C.memmove(handle, bytes([rank]) * 64, 64)
            return 0
        return 7  # PB_ERR_UNAVAILABLE

    def pb_peer_import(self, ctx, dev, world, handles):
        self.calls.append(("import", world, bytes(handles)))
        return 0

    def pb_peer_close(self, ctx, dev):
        self.calls.append(("peer_close",))
        return 0


class FakeBackend:
    def __init__(self, all_export=False):
        self._lib = FakeCommLib(all_export)
        self._ctx = C.c_void_p(1)
        self._lock = threading.RLock()


def _worker(rank, world, port, scenario, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    try:
        if scenario == "partition":
            got = {}
            for n in (0, 1, 7, 8, 16384, 65539):
                got[n] = shard_range(n, rank, world)
            gathered = [None] * world
            dist.all_gather_object(gathered, got)
            queue.put((rank, gathered))
        elif scenario in ("rendezvous", "mailboxes"):
            backend = FakeBackend(all_export=scenario == "mailboxes")
            group = Group(backend, rank, world, store, prefix="t1", timeout=10)
            backend._lib.calls.append(("p2p", group.p2p))
            group.heartbeat()
            group.heartbeat()
            group.close()
            queue.put((rank, backend._lib.calls))
        elif scenario == "failure":
            backend = FakeBackend()
            group = Group(backend, rank, world, store, prefix="t2", timeout=3)
            group.heartbeat()  # step 0: everyone present
            dist.barrier()
            if rank == 1:
                queue.put((rank, "left"))
                return  # leaves between steps, nothing in flight
            t0 = time.monotonic()
            try:
                with group:
                    group.heartbeat()  # step 1: rank 1 never arrives
                queue.put((rank, "no failure detected"))
            except RankFailure:
                queue.put((rank, ("detected", time.monotonic() - t0, backend._lib.calls)))
    finally:
        if scenario != "failure":
            dist.destroy_process_group()


def _run(scenario, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_shard_range_single_process():
    for n in (0, 1, 5, 8, 100, 65539):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_partition_is_disjoint_and_complete_across_ranks():
    results = _run("partition")
    for gathered in results.values():
        for n in gathered[0]:
            spans = [g[n] for g in gathered]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert spans[0][1] == spans[1][0]


def test_nccl_id_rendezvous_through_the_store():
    results = _run("rendezvous")
    inits = {r: [c for c in calls if c[0] == "init"] for r, calls in results.items()}
    assert all(len(v) == 1 for v in inits.values())
    (_, w0, r0, id0), (_, w1, r1, id1) = inits[0][0], inits[1][0]
    assert (w0, r0, w1, r1) == (2, 0, 2, 1)
    assert id0 == id1 == bytes(range(128))
    assert ("uid",) in results[0] and ("uid",) not in results[1]
    assert all(calls[-1] == ("destroy",) for calls in results.values())
    # Rank 1 could not export a mailbox: both ranks agree on the NCCL path,
    # and rank 0 unmaps what it had set up before the group is used.
    assert all(("p2p", False) in calls for calls in results.values())
    assert results[0].index(("peer_close",)) < results[0].index(("p2p", False))


def test_four_ranks_partition_and_fall_back_together():
    """Four ranks: contiguous shards, one shared NCCL id, and rank 1's failed
    mailbox export sends every rank to the NCCL path."""
    parts = _run("partition", world=4)
    for gathered in parts.values():
        for n in gathered[0]:
            spans = [g[n] for g in gathered]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    results = _run("rendezvous", world=4)
    inits = {r: [c for c in calls if c[0] == "init"] for r, calls in results.items()}
    assert sorted((c[0][1], c[0][2]) for c in inits.values()) == [(4, r) for r in range(4)]
    assert len({c[0][3] for c in inits.values()}) == 1
    assert all(("p2p", False) in calls for calls in results.values())


def test_four_ranks_map_every_mailbox_in_rank_order():
    """Every rank exports: each imports the four handles concatenated in rank
    order and the group uses the peer mailboxes."""
    results = _run("mailboxes", world=4)
    want = b"".join(bytes([r]) * 64 for r in range(4))
    for calls in results.values():
        imports = [c for c in calls if c[0] == "import"]
        assert imports == [("import", 4, want)]
        assert ("p2p", True) in calls


def test_departed_rank_is_detected_before_any_collective():
    results = _run("failure")
    assert results[1] == "left"
    outcome = results[0]
    assert outcome[0] == "detected", outcome
    elapsed, calls = outcome[1], outcome[2]
    assert 2.5 <= elapsed < 30
    # The survivor aborted its communicator instead of waiting on the peer.
    assert calls[-1] == ("abort",)
