"""Builds the engine's shared library in-tree with nvcc for sm_100a, and the
sidecar server (a plain C++ program over the library's C ABI).

``python -m cruise_b200.build`` writes ``cruise_b200/libcruise_epoch.so`` and
``cruise_b200/cruise_epoch_server``.  nvcc cross-compiles without a GPU, so this
runs on any host with CUDA 12.9.
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
SERVER = PACKAGE / "cruise_epoch_server"
SOURCES = [CSRC / "engine.cu"]
SERVER_SOURCES = [CSRC / "sidecar_server.cpp"]
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


def _fresh(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return False
    built = target.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources + HEADERS)


def up_to_date() -> bool:
    return _fresh(LIBRARY, SOURCES) and _fresh(SERVER, SERVER_SOURCES + [LIBRARY])


def build_server() -> Path:
    """The sidecar server, linked against the in-tree library (found next to it)."""
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("a C++ compiler (g++) is required to build the sidecar server")
    tmp = SERVER.with_name(f"{SERVER.name}.tmp{os.getpid()}")
    cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-o", str(tmp), *map(str, SERVER_SOURCES),
           f"-L{PACKAGE}", "-l:libcruise_epoch.so", "-Wl,-rpath,$ORIGIN"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, SERVER)
    return SERVER


def link_flags() -> list[str]:
    """No library beyond the CUDA runtime (linked statically by nvcc); the
    driver's tensor-map encoder is found at run time through the runtime."""
    return []


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIBRARY
    if force or not _fresh(LIBRARY, SOURCES):
        tmp = LIBRARY.with_suffix(f".so.tmp{os.getpid()}")
        cmd = [nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-o", str(tmp), *map(str, SOURCES),
               *link_flags()]
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIBRARY)
    build_server()
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
