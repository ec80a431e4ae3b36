"""Stable identity for sm100 kernel measurements and deployments.

Mirrors the reference's ``deployment/environment.py`` (``ImplementationScope``
:23-27, ``stable_digest`` :40-44, ``solution_implementation_digest`` :75-96,
``EnvironmentFingerprint`` :150-296).  The Triton version of the reference's
fingerprint becomes the libb200tx ABI version, and the implementation digest
covers the CUDA sources of the kernels plus the Python that launches them.
The driver version is read through NVML instead of spawning ``nvidia-smi``.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from enum import StrEnum
from functools import lru_cache
from pathlib import Path
from typing import Any

import torch

PACKAGE_ROOT = Path(__file__).resolve().parents[1]


class ImplementationScope(StrEnum):
    """Resident and streamed lifecycles, versioned independently."""

    RESIDENT = "resident"
    SHAPE14 = "shape14"


def _stable_json(value: object) -> bytes:
    return json.dumps(
        value, ensure_ascii=False, sort_keys=True, separators=(",", ":"), allow_nan=False
    ).encode("utf-8")


def stable_digest(value: object) -> str:
    """One canonical SHA-256 identity for JSON-compatible data."""

    return hashlib.sha256(_stable_json(value)).hexdigest()


def _scope_sources(root: Path, scope: ImplementationScope) -> list[Path]:
    sources = sorted((root / "csrc").glob("*.cu*"))
    sources += sorted((root / "solution" / "kernels").glob("*.py"))
    sources += sorted((root / "solution" / "runtimes").glob("*.py"))
    sources += [root / "solution" / "transformer.py", root / "solution" / "_native.py"]
    if scope is ImplementationScope.SHAPE14:
        sources += sorted((root / "solution" / "shape14").glob("*.py"))
    return [path for path in sources if path.exists()]


def solution_implementation_digest(
    package_root: Path = PACKAGE_ROOT, *, scope: ImplementationScope = ImplementationScope.RESIDENT
) -> str:
    """Digest of the kernel sources and launch code in the requested scope."""

    root = Path(package_root)
    records = [
        {"path": path.relative_to(root).as_posix(), "sha256": hashlib.sha256(path.read_bytes()).hexdigest()}
        for path in _scope_sources(root, ImplementationScope(scope))
    ]
    return stable_digest(records)


@lru_cache(maxsize=16)
def _driver_version(index: int) -> str:
    try:
        import pynvml  # nvidia-ml-py

        pynvml.nvmlInit()
        try:
            version = pynvml.nvmlSystemGetDriverVersion()
        finally:
            pynvml.nvmlShutdown()
        return version.decode() if isinstance(version, bytes) else str(version)
    except Exception:  # noqa: BLE001 - NVML absent or not permitted
        return "unknown"


def kernel_library_version() -> str:
    from solution import _native

    try:
        lib = _native.load()
    except RuntimeError:
        return "unavailable"
    return f"abi-{lib.b200tx_abi_version()}"


def _required_string(value: object, name: str) -> str:
    if not isinstance(value, str) or not value:
        raise ValueError(f"environment fingerprint field {name!r} must be a string")
    return value


@dataclass(frozen=True, slots=True)
class EnvironmentFingerprint:
    """Execution facts that may change a kernel-variant winner."""

    device_name: str
    compute_capability: str
    driver_version: str
    torch_version: str
    cuda_runtime_version: str
    kernel_library_version: str
    solution_implementation_digest: str
    scope: ImplementationScope = ImplementationScope.RESIDENT

    @classmethod
    def detect(
        cls,
        device: str | torch.device,
        *,
        package_root: Path = PACKAGE_ROOT,
        scope: ImplementationScope = ImplementationScope.RESIDENT,
    ) -> EnvironmentFingerprint:
        resolved = torch.device(device)
        if resolved.type != "cuda" or not torch.cuda.is_available():
            raise ValueError("environment fingerprint detection requires CUDA")
        index = torch.cuda.current_device() if resolved.index is None else resolved.index
        major, minor = torch.cuda.get_device_capability(index)
        runtime = torch.version.cuda
        if not runtime:
            raise RuntimeError("CUDA runtime version is unavailable from PyTorch")
        normalized = ImplementationScope(scope)
        return cls(
            device_name=torch.cuda.get_device_name(index),
            compute_capability=f"{major}.{minor}",
            driver_version=_driver_version(index),
            torch_version=str(torch.__version__),
            cuda_runtime_version=str(runtime),
            kernel_library_version=kernel_library_version(),
            solution_implementation_digest=solution_implementation_digest(
                package_root, scope=normalized
            ),
            scope=normalized,
        )

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> EnvironmentFingerprint:
        return cls(
            device_name=_required_string(value["device_name"], "device_name"),
            compute_capability=_required_string(value["compute_capability"], "compute_capability"),
            driver_version=_required_string(value["driver_version"], "driver_version"),
            torch_version=_required_string(value["torch_version"], "torch_version"),
            cuda_runtime_version=_required_string(value["cuda_runtime_version"], "cuda_runtime_version"),
            kernel_library_version=_required_string(
                value["kernel_library_version"], "kernel_library_version"
            ),
            solution_implementation_digest=_required_string(
                value["solution_implementation_digest"], "solution_implementation_digest"
            ),
            scope=ImplementationScope(_required_string(value["scope"], "scope")),
        )

    def to_dict(self) -> dict[str, str]:
        return {
            "scope": self.scope.value,
            "device_name": self.device_name,
            "compute_capability": self.compute_capability,
            "driver_version": self.driver_version,
            "torch_version": self.torch_version,
            "cuda_runtime_version": self.cuda_runtime_version,
            "kernel_library_version": self.kernel_library_version,
            "solution_implementation_digest": self.solution_implementation_digest,
        }

    @property
    def identity(self) -> str:
        """Identity of this exact executable environment, sources included."""

        return stable_digest(self.to_dict())

    @property
    def measurement_identity(self) -> str:
        """Hardware/runtime identity, independent of the measured source version."""

        value = self.to_dict()
        value.pop("solution_implementation_digest")
        return stable_digest(value)


__all__ = [
    "EnvironmentFingerprint",
    "ImplementationScope",
    "kernel_library_version",
    "solution_implementation_digest",
    "stable_digest",
]
