"""Builds the engine's shared library in-tree with nvcc for sm_100a.

``python -m cruise_b200.build`` writes ``cruise_b200/libcruise_epoch.so``.
nvcc cross-compiles without a GPU, so this runs on any host with CUDA 12.9.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libcruise_epoch.so"
SOURCES = [CSRC / "engine.cu"]
HEADERS = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((PACKAGE.parent / "include").glob("*.h"))
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build the engine")
    return found


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-o", str(tmp), *map(str, SOURCES)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
