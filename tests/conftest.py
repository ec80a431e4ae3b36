"""Shared test setup.

* Registers the ``gpu`` marker: tests that launch libb200tx kernels carry it
  and are skipped when no CUDA device is visible.
* Puts the package directory (which holds the ``solution`` and ``deployment``
  packages, mirroring the reference's module names) and the repository root
  (for ``oracle``) on ``sys.path``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
PACKAGE_DIR = REPO / "ml-guided-program-search-for-shape-specialized-transformer-optimization_b200"
GOLDEN = REPO / "tests" / "golden"
for path in (str(PACKAGE_DIR), str(REPO)):
    if path not in sys.path:
        sys.path.insert(0, path)

# Tolerances of the parity gate: bf16 compute against the reference's fp32.
MAX_ABS_TOL = 2e-2
REL_L2_TOL = 1e-2


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device and libb200tx")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {key: data[key] for key in data.files}


def parity_errors(got: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = got - ref
    max_abs = float(np.abs(diff).max()) if diff.size else 0.0
    denom = float(np.linalg.norm(ref))
    rel = float(np.linalg.norm(diff) / denom) if denom > 0 else float(np.linalg.norm(diff))
    return max_abs, rel
