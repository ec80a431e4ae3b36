"""Install the reference's Python packages into baseline/_ref (git-ignored).

The reference repository has no setup.py or pyproject.toml, so it cannot be
pip-installed as it stands.  This copies it to a temporary directory, adds a
minimal pyproject.toml that lists its ``official``, ``solution`` and
``deployment`` packages (with their JSON data), and installs that copy
offline, without dependencies, into ``baseline/_ref``.  ``bench.py`` imports
the reference's own CPU forward (``official.BaselineTransformer``) from there
for its ``cpu_baseline`` leg and its ``--impl reference`` arm.

usage: python baseline/install_reference.py REFERENCE_ROOT
"""

from __future__ import annotations

import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

TARGET = Path(__file__).resolve().parent / "_ref"

PYPROJECT = """\
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "shape-aware-transformer-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
include = ["official*", "solution*", "deployment*"]

[tool.setuptools.package-data]
"*" = ["*.json"]
"""


def install(reference_root: Path) -> None:
    if not (reference_root / "official" / "torch_transformer_benchmark.py").exists():
        raise SystemExit(f"{reference_root} does not hold the reference's official/ package")
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "reference"
        shutil.copytree(reference_root, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        (copy / "pyproject.toml").write_text(PYPROJECT)
        if TARGET.exists():
            shutil.rmtree(TARGET)
        subprocess.run(
            [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
             "--target", str(TARGET), str(copy)],
            check=True,
        )
    print(f"installed the reference into {TARGET}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python baseline/install_reference.py REFERENCE_ROOT")
    install(Path(sys.argv[1]).resolve())
