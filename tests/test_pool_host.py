"""Host logic of the single-process GPU pool (``device="0-7"``): device lists,
block plans, the split decision on BASELINE's shapes, and the order of the
copies, waits and launches the split product queues (against a recording
stand-in for the library, no GPU)."""

from __future__ import annotations

import ctypes as C

import pytest

from pacho_b200 import _lib, pool


def test_parse_devices():
    assert pool.parse_devices(None) == [0]
    assert pool.parse_devices(3) == [3]
    assert pool.parse_devices("5") == [5]
    assert pool.parse_devices("cuda:2") == [2]
    assert pool.parse_devices("0-7") == list(range(8))
    assert pool.parse_devices("0, 2,5") == [0, 2, 5]
    assert pool.parse_devices("1-2,6") == [1, 2, 6]
    assert pool.parse_devices(None, gpus=4) == [0, 1, 2, 3]
    assert pool.parse_devices("4", gpus=2) == [4, 5]
    assert pool.parse_devices("0-1", gpus=2) == [0, 1]
    for bad in ("a", "3-1", "0,0", "-1", "0-1x"):
        with pytest.raises(ValueError):
            pool.parse_devices(bad)
    with pytest.raises(ValueError):
        pool.parse_devices("0-3", gpus=2)
    with pytest.raises(ValueError):
        pool.parse_devices(None, gpus=0)


@pytest.mark.parametrize("total,parts,align", [(16384, 8, 128), (1000, 8, 128), (8, 8, 1), (3, 8, 1),
                                               (1, 2, 128), (129, 2, 128), (7, 3, 1), (0, 4, 1)])
def test_blocks_cover_the_range_in_order(total, parts, align):
    got = pool.blocks(total, parts, align)
    assert len(got) <= parts
    if not total:
        assert got == []
        return
    assert [lo for lo, _ in got] == [0] + [hi for _, hi in got[:-1]]
    assert (got[-1][1] if got else 0) == total
    assert all(hi > lo for lo, hi in got)
    assert all(lo % align == 0 for lo, _ in got)
    sizes = [hi - lo for lo, hi in got]
    if len(got) > 1:
        # Equal up to one alignment unit, except a short last block.
        assert max(sizes[:-1]) - min(sizes[:-1]) <= align


def test_plan_layouts():
    two_d = pool.plan((4096, 512), (512, 256), (), 4096, 256, 512)
    assert (two_d.outer, two_d.a_block, two_d.b_block, two_d.c_block, two_d.b_whole) == (4096, 512, 0, 256,
                                                                                          512 * 256)
    shared_b = pool.plan((8, 16, 512, 256), (1, 16, 256, 384), (8, 16), 512, 384, 256)
    assert shared_b is None  # B batched along the inner dimension only: no contiguous cut
    batched = pool.plan((8, 16, 512, 256), (8, 16, 256, 384), (8, 16), 512, 384, 256)
    assert (batched.outer, batched.a_block, batched.b_block, batched.c_block) == (
        8, 16 * 512 * 256, 16 * 256 * 384, 16 * 512 * 384)
    whole_b = pool.plan((8, 512, 256), (256, 384), (8,), 512, 384, 256)
    assert (whole_b.outer, whole_b.b_block, whole_b.b_whole) == (8, 0, 256 * 384)
    assert pool.plan((512, 256), (8, 256, 384), (8,), 512, 384, 256) is None  # A broadcast


def test_split_decision_on_baseline_shapes():
    f32, f64 = 4, 8
    # Config 5: 16384^3 float32 and 8192^3 float64 split over 8 GPUs.
    assert pool.worth_splitting(2.0 * 16384 ** 3, f32, 16384 ** 2 * 4, 16384 ** 2 * 4, 16384 ** 2 * 4, 8)
    assert pool.worth_splitting(2.0 * 8192 ** 3, f64, 8192 ** 2 * 8, 8192 ** 2 * 8, 8192 ** 2 * 8, 8)
    # Config 1 (1024^3) and config 3 (12.9 GFLOP) stay on one GPU.
    assert not pool.worth_splitting(2.0 * 1024 ** 3, f32, 4 << 20, 4 << 20, 4 << 20, 8)
    assert not pool.worth_splitting(2.0 * 8 * 16 * 512 * 256 * 384, f32, 8 * 16 * 512 * 256 * 4,
                                    16 * 256 * 384 * 4, 8 * 16 * 512 * 384 * 4, 8)
    assert not pool.worth_splitting(2.0 * 16384 ** 3, f32, 1, 1, 1, 1)


class FakeLib:
    """Records the pool's library calls; pointers are distinct integers."""

    def __init__(self):
        self.calls = []
        self.next = 1 << 40

    def pb_peer_enable(self, ctx, flag):
        flag._obj.value = 1
        return 0

    def pb_alloc_mapped(self, ctx, dev, nbytes, ptr):
        self.next += 1 << 32
        ptr._obj.value = self.next
        self.calls.append(("alloc", dev, nbytes, self.next))
        return 0

    def pb_free_mapped(self, ctx, dev, ptr):
        self.calls.append(("free", dev, ptr.value))
        return 0

    def pb_sync(self, ctx, dev):
        self.calls.append(("sync", dev))
        return 0

    def pb_stream_wait(self, ctx, waiter, waiter_stream, signal, signal_stream):
        self.calls.append(("wait", waiter, waiter_stream, signal, signal_stream))
        return 0

    def pb_copy_peer(self, ctx, dst_dev, dst, src_dev, src, nbytes, on, stream):
        self.calls.append(("copy", dst_dev, dst.value, src_dev, src.value, nbytes, on, stream))
        return 0


class FakeBackend:
    def __init__(self):
        self._lib, self._ctx = FakeLib(), C.c_void_p(1)


def _run(dp, be, sp, A, B, O, isz):
    def gemm(dev, outer, pa, pb, pc):
        be._lib.calls.append(("gemm", dev, outer, pa, pb, pc))

    dp.matmul(_lib.PB_F32, isz, sp, A, B, O, gemm)


@pytest.mark.parametrize("ndev", [2, 3, 8])
def test_split_product_queues_copies_waits_and_launches_in_order(ndev, monkeypatch):
    monkeypatch.setattr(pool, "CHUNK_BYTES", 1 << 20)
    be = FakeBackend()
    dp = pool.DevicePool(be, ndev)
    assert dp.all_peer
    M, N, K, isz = 1000, 96, 640, 4
    sp = pool.plan((M, K), (K, N), (), M, N, K)
    A, B, O = 1 << 20, 2 << 30, 3 << 30
    _run(dp, be, sp, A, B, O, isz)
    calls = be._lib.calls
    parts = pool.blocks(M, ndev, pool.ROW_ALIGN)
    used = len(parts)
    allocs = [c for c in calls if c[0] == "alloc"]
    ws = {(c[1], role): c[3] for c, role in zip(allocs, ["a", "b", "c"] * used)}
    assert len(allocs) == 3 * (used - 1) and all(c[1] >= 1 for c in allocs)
    work = [c for c in calls if c[0] != "alloc"]
    # Every stream first waits for the primary's kernel stream.
    head = [("wait", 0, 1, 0, 0)] + [w for d in range(1, used) for w in (("wait", d, 0, 0, 0), ("wait", d, 1, 0, 0))]
    assert work[: len(head)] == head
    copies = [c for c in work if c[0] == "copy"]
    assert all(c[7] == 1 for c in copies)  # every copy on a copy stream
    # The primary pushes the A blocks into the mapped workspaces.
    for d, (lo, hi) in enumerate(parts[1:], start=1):
        assert ("copy", d, ws[(d, "a")], 0, A + lo * K * isz, (hi - lo) * K * isz, 0, 1) in copies
    # B down the chain in chunks, each forwarded by the device before.
    total = K * N * isz
    chunks = -(-total // pool.CHUNK_BYTES)
    chain = [c for c in copies if c[1] != 0 and c[3] == c[1] - 1 and
             (c[3] == 0 and B <= c[4] < B + total or c[3] > 0 and ws[(c[3], "b")] <= c[4] < ws[(c[3], "b")] + total)]
    assert len(chain) == chunks * (used - 1)
    assert all(c[6] == c[3] and ws[(c[1], "b")] <= c[2] < ws[(c[1], "b")] + total for c in chain)
    # A hop from d - 1 comes after d - 1's copy stream joined d - 2's.
    for c in chain:
        if c[3] >= 1:
            i = work.index(c)
            assert ("wait", c[3], 1, c[3] - 1, 1) in work[:i]
    # Blocks: the other devices first, the primary last, each with its rows;
    # each device's kernel stream joined its suppliers before any block.
    launches = [c for c in work if c[0] == "gemm"]
    assert [(c[1], c[2]) for c in launches] == [(d, hi - lo) for d, (lo, hi) in enumerate(parts)][1:] + [
        (0, parts[0][1] - parts[0][0])]
    assert launches[-1][3:] == (A, B, O)
    first_gemm = work.index(launches[0])
    for d in range(1, used):
        assert ("wait", d, 0, 0, 1) in work[:first_gemm]
        if d > 1:
            assert ("wait", d, 0, d - 1, 1) in work[:first_gemm]
    # After the first block only the primary's streams wait.
    assert all(c[1] == 0 for c in work[first_gemm:] if c[0] == "wait")
    # The primary pulls each C block on its copy stream after joining that
    # device's kernel stream, and its kernel stream ends after everything.
    for d, (lo, hi) in enumerate(parts[1:], start=1):
        pull = ("copy", 0, O + lo * N * isz, d, ws[(d, "c")], (hi - lo) * N * isz, 0, 1)
        i = work.index(pull)
        assert ("wait", 0, 1, d, 0) in work[first_gemm:i]
    tail = work[-(1 + 2 * (used - 1)):]
    assert tail[0] == ("wait", 0, 0, 0, 1)
    assert all(("wait", 0, 0, d, 0) in tail and ("wait", 0, 0, d, 1) in tail for d in range(1, used))
    assert dp.splits == 1
    # A second product of the same shape reuses the workspaces.
    n_alloc = len(allocs)
    _run(dp, be, sp, A, B, O, isz)
    assert len([c for c in be._lib.calls if c[0] == "alloc"]) == n_alloc
    assert not [c for c in be._lib.calls if c[0] == "free"]
    dp.close()
    assert sorted(c[2] for c in be._lib.calls if c[0] == "free") == sorted(c[3] for c in allocs)


def test_growing_a_workspace_waits_for_every_device_first():
    be = FakeBackend()
    dp = pool.DevicePool(be, 2)
    small = pool.plan((256, 64), (64, 64), (), 256, 64, 64)
    big = pool.plan((4096, 64), (64, 64), (), 4096, 64, 64)
    _run(dp, be, small, 1 << 20, 2 << 20, 3 << 20, 4)
    be._lib.calls.clear()
    _run(dp, be, big, 1 << 20, 2 << 20, 3 << 20, 4)
    calls = be._lib.calls
    first_free = next(i for i, c in enumerate(calls) if c[0] == "free")
    assert {("sync", 0), ("sync", 1)} <= set(calls[:first_free])


def test_split_ends_the_primary_after_every_device_when_a_launch_fails():
    be = FakeBackend()
    dp = pool.DevicePool(be, 4)
    sp = pool.plan((1024, 64), (64, 64), (), 1024, 64, 64)

    def gemm(dev, *args):
        if dev == 2:
            raise RuntimeError("launch failed")

    with pytest.raises(RuntimeError):
        dp.matmul(_lib.PB_F32, 4, sp, 1 << 20, 2 << 20, 3 << 20, gemm)
    waits = [c for c in be._lib.calls if c[0] == "wait"]
    assert ("wait", 0, 0, 0, 1) in waits
    assert all(("wait", 0, 0, d, 0) in waits and ("wait", 0, 0, d, 1) in waits for d in range(1, 4))
    assert dp.splits == 0
