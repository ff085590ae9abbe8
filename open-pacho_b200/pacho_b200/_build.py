"""Build libpacho_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m pacho_b200._build [--force] [--verbose]`` from the
``open-pacho_b200`` directory, or ``pacho_b200._build.build()``.  Objects go to
``open-pacho_b200/_build``; the shared library lands next to this file so it
travels with the source tree.  The CUDA runtime is linked statically, so the
library loads (and reports "no device") on machines without a GPU driver.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent  # open-pacho_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
BUILD = ROOT / "_build"
LIBRARY = PKG / "libpacho_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the B200 backend must be compiled with CUDA 12.8+")
    return found


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(nvcc: str, src: Path, headers: list[Path], force: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if not force and not _stale(obj, [src, *headers]):
        return obj, ""
    cmd = [nvcc, *ARCH, *CFLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source and link the shared library; returns its path."""
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(lambda s: _compile(nvcc, s, headers, force), sources))
    objects = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if force or _stale(LIBRARY, objects):
        cmd = [
            nvcc,
            *ARCH,
            "-shared",
            "-cudart",
            "static",
            "-o",
            str(LIBRARY),
            *map(str, objects),
            "-Xlinker",
            "--no-undefined",
            "-ldl",
            "-lpthread",
            "-lrt",
        ]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    return LIBRARY


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
