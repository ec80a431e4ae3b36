"""The C ABI as a C program sees it: include/b200tx.h compiles as strict C99
and a C consumer linked against libb200tx gets the documented status codes
and messages (tests/c_abi/abi_consumer.c).  Needs gcc and the built library,
no GPU."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from solution import _native

REPO = Path(__file__).resolve().parents[1]
CUDA_INCLUDE = Path("/usr/local/cuda/include")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc is not installed")
def test_header_compiles_as_c99_and_a_c_consumer_links_and_runs(tmp_path: Path) -> None:
    lib = _native.library_path()
    if not lib.exists():
        pytest.skip("libb200tx.so is not built")
    exe = tmp_path / "abi_consumer"
    cmd = [
        "gcc", "-std=c99", "-Wall", "-Wextra", "-Werror",
        "-I", str(REPO / "include"), "-I", str(CUDA_INCLUDE),
        str(REPO / "tests" / "c_abi" / "abi_consumer.c"),
        "-L", str(lib.parent), "-l:" + lib.name, f"-Wl,-rpath,{lib.parent}",
        "-o", str(exe),
    ]
    built = subprocess.run(cmd, capture_output=True, text=True, check=False)
    assert built.returncode == 0, built.stderr
    ran = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60, check=False)
    assert ran.returncode == 0, ran.stderr
    assert ran.stdout.splitlines() == [f"abi {_native.ABI_VERSION}", "ok"]
