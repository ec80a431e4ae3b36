"""Build libb200tx.so (the sm_100a kernels and their C ABI) in-tree.

The library is compiled from ``csrc/b200tx.cu`` (which includes the kernel
headers next to it) with nvcc for ``sm_100a`` only and written to
``solution/_lib/libb200tx.so``, where :mod:`solution._native` loads it.
Run ``python build_native.py`` or call :func:`build`.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"
LIB_DIR = PACKAGE_DIR / "solution" / "_lib"
LIB_PATH = LIB_DIR / "libb200tx.so"

NVCC_FLAGS = (
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
)


def _nvcc() -> str:
    candidates = [
        os.environ.get("NVCC"),
        shutil.which("nvcc"),
        "/usr/local/cuda/bin/nvcc",
    ]
    for candidate in candidates:
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu")) + sorted(CSRC_DIR.glob("*.cuh")) + [
        INCLUDE_DIR / "b200tx.h"
    ]


def is_stale() -> bool:
    """Return whether the library is missing or older than any source file."""

    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(source.stat().st_mtime > built for source in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or stale; return its path."""

    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    command = [
        _nvcc(),
        *NVCC_FLAGS,
        f"-I{INCLUDE_DIR}",
        "-o",
        str(tmp),
        str(CSRC_DIR / "b200tx.cu"),
    ]
    if verbose:
        print(" ".join(command), flush=True)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(
            "nvcc failed building libb200tx.so:\n" + result.stdout + result.stderr
        )
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
