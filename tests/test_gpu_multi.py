"""Sharded paths on 2 and 4 GPUs (child processes under torchrun; skipped
without enough GPUs).

NVLS is off (NCCL_NVLS_ENABLE=0) and the library's communicator waits are
bounded (PB_COMM_TIMEOUT_S); the whole launch runs in its own process group
with a hard timeout.  The departed-rank case leaves only between steps, with
nothing in flight, and is detected on the host.
"""

from __future__ import annotations

import ctypes as C
import json
import os
import signal
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _gpu_count() -> int:
    from pacho_b200 import _lib

    n = C.c_int(0)
    return n.value if _lib.load().pb_device_count(C.byref(n)) == 0 else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(failure: bool, tmp_path, nproc: int = 2, timeout_case: bool = False):
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0", "PB_COMM_TIMEOUT_S": "60",
           "PB_STORE_PORT": str(_free_port()), "PB_TEST_FAILURE": "1" if failure else "0",
           "PB_TEST_TIMEOUT": "1" if timeout_case else "0", "PB_RESULT_DIR": str(tmp_path)}
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "multigpu_worker.py")]
    proc = subprocess.Popen(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE,
                            stderr=subprocess.STDOUT, text=True, start_new_session=True)
    try:
        out, _ = proc.communicate(timeout=400)
    except subprocess.TimeoutExpired:
        os.killpg(proc.pid, signal.SIGKILL)
        out, _ = proc.communicate()
        pytest.fail(f"{nproc}-GPU worker timed out:\n" + out[-4000:])
    assert proc.returncode == 0, out[-4000:]
    files = sorted(tmp_path.glob("rank*.json"))
    assert len(files) == nproc, out[-4000:]
    results = [json.loads(f.read_text()) for f in files]
    return {r["rank"]: r for r in results}


@pytest.mark.parametrize("nproc", [2, 4, 8])
def test_sharded_paths(tmp_path, nproc):
    """Sharded norm and DOT through peer mailboxes of nproc slots (both
    parities), row blocks and the batch split with uneven shards, gathers."""
    if _gpu_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    results = _launch(failure=False, tmp_path=tmp_path, nproc=nproc)
    assert sorted(results) == list(range(nproc))
    for r in results.values():
        checks = {k: v for k, v in r.items() if k != "rank"}
        assert checks and all(v == 0 for v in checks.values()), r


def test_mailbox_wait_runs_out_and_reports_on_two_gpus(tmp_path):
    """A peer that never pushes: the merge kernel's bounded wait (100 ms here)
    runs out, the kernel returns, pb_sync reports PB_ERR_DEVICE and the
    context keeps working."""
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    results = _launch(failure=False, tmp_path=tmp_path, timeout_case=True)
    r0 = results[0]
    if r0.get("p2p_unavailable"):
        pytest.skip("peer mailboxes unavailable (NCCL fallback in use)")
    assert r0["timeout_submit_status"] == 0
    assert r0["timeout_sync_status"] == 6  # PB_ERR_DEVICE
    assert 0.1 <= r0["timeout_seconds"] < 5.0
    assert r0["after_timeout_dot"] == 0


def test_departed_rank_is_detected_on_two_gpus(tmp_path):
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    results = _launch(failure=True, tmp_path=tmp_path)
    assert results[1].get("left") is True
    assert results[0]["failure"] == "detected", results[0]
    assert 4.5 <= results[0]["failure_seconds"] < 60
