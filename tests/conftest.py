"""Shared test setup.

``-m gpu`` tests need a B200 and fail (never skip) when the CUDA library or the
device is missing; ``-m "not gpu"`` tests run on any CPU machine.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "open-pacho_b200", ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"

# OpenPacho's own front end (the reference) for the CPU integration tests:
# importable when installed, or from a source tree named by OPENPACHO_SRC
# (the directory that contains the ``openpacho`` package).  Those tests skip
# without it; the GPU machines do not have it.
_OPENPACHO_SRC = os.environ.get("OPENPACHO_SRC")
if _OPENPACHO_SRC and _OPENPACHO_SRC not in sys.path:
    sys.path.append(_OPENPACHO_SRC)


@pytest.fixture(scope="session")
def openpacho():
    return pytest.importorskip("openpacho", reason="OpenPacho not importable (set OPENPACHO_SRC)")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    data = np.load(GOLDEN / "golden.npz")
    meta = json.loads((GOLDEN / "golden.json").read_text())["cases"]
    return data, meta


@pytest.fixture(scope="session")
def b200():
    """The b200 backend on device 0 (hard failure if unavailable)."""
    from pacho_b200 import B200Backend

    backend = B200Backend(0)
    yield backend
    backend.synchronize()
