"""Builds the sm_100a shared library `libdory_decode.so` next to this file.

The library is plain C ABI (include/dory_decode.h) linked against the CUDA runtime only;
the Python host code loads it with ctypes, so no torch headers are involved and the same
.so serves a C, C++ or Python caller.  Run `python build_native.py` or call `build()`.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = [HERE / "csrc" / "dory_decode.cu"]
HEADERS = [ROOT / "include" / "dory_decode.h"]
LIBRARY = HERE / "libdory_decode.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--cudart", "shared",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library if a source is newer than it; returns its path."""
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-o", str(tmp),
           *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
