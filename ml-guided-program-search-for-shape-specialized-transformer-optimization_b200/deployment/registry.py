"""Exact-match registry of selected configurations per (environment, shape).

Mirrors the reference's ``deployment/registry.py`` (``ShapeFingerprint``
:20-60, ``resolve_deployed_config`` :107-121, ``iter_deployed_configs``
:124-148, ``publish_deployed_config`` :151-205): a JSON document of bundles,
one per hardware measurement identity, each holding shape -> ConfigSpec
entries.  Lookups are exact; a miss returns ``None`` and the caller falls back
to the default sm100 program.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from solution.config import ConfigSpec

from .environment import EnvironmentFingerprint

DEFAULT_DEPLOYED_CONFIGS_PATH = Path(__file__).resolve().parent / "deployed_configs.json"
DEPLOYMENT_SCHEMA_VERSION = 4


@dataclass(frozen=True, slots=True)
class ShapeFingerprint:
    batch_size: int
    qkv_dim: int
    heads: int
    seq_len: int
    layers: int
    causal: bool
    ffn_dim: int
    dtype: str
    padding_ratio: float
    input_scale: float

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> ShapeFingerprint:
        return cls(
            batch_size=int(value["batch_size"]),
            qkv_dim=int(value["qkv_dim"]),
            heads=int(value["heads"]),
            seq_len=int(value["seq_len"]),
            layers=int(value["layers"]),
            causal=bool(value["causal"]),
            ffn_dim=int(value["ffn_dim"]),
            dtype=str(value["dtype"]),
            padding_ratio=float(value["padding_ratio"]),
            input_scale=float(value["input_scale"]),
        )

    def to_dict(self) -> dict[str, Any]:
        return {
            "batch_size": self.batch_size,
            "qkv_dim": self.qkv_dim,
            "heads": self.heads,
            "seq_len": self.seq_len,
            "layers": self.layers,
            "causal": self.causal,
            "ffn_dim": self.ffn_dim,
            "dtype": self.dtype,
            "padding_ratio": self.padding_ratio,
            "input_scale": self.input_scale,
        }


def _load(path: str | Path) -> dict[str, Any]:
    value = json.loads(Path(path).read_text(encoding="utf-8"))
    if not isinstance(value, dict) or not isinstance(value.get("bundles"), list):
        raise ValueError("deployed config file must contain a bundles array")
    return value


def _keys(
    hardware: EnvironmentFingerprint | dict[str, Any], shape: ShapeFingerprint | dict[str, Any]
) -> tuple[EnvironmentFingerprint, ShapeFingerprint]:
    return (
        hardware if isinstance(hardware, EnvironmentFingerprint) else EnvironmentFingerprint.from_dict(hardware),
        shape if isinstance(shape, ShapeFingerprint) else ShapeFingerprint.from_dict(shape),
    )


def _matching_entries(*, hardware: EnvironmentFingerprint, path: str | Path) -> tuple[dict[str, Any], ...]:
    try:
        document = _load(path)
    except FileNotFoundError:
        return ()
    if document.get("schema_version") != DEPLOYMENT_SCHEMA_VERSION:
        return ()
    for bundle in document["bundles"]:
        if not isinstance(bundle, dict) or not isinstance(bundle.get("hardware"), dict):
            continue
        persisted = EnvironmentFingerprint.from_dict(bundle["hardware"])
        if persisted.measurement_identity == hardware.measurement_identity:
            return tuple(entry for entry in bundle.get("entries", []) if isinstance(entry, dict))
    return ()


def resolve_deployed_config(
    *,
    hardware: EnvironmentFingerprint | dict[str, Any],
    shape: ShapeFingerprint | dict[str, Any],
    path: str | Path = DEFAULT_DEPLOYED_CONFIGS_PATH,
) -> ConfigSpec | None:
    """The exact device/shape config, or ``None`` when none was measured."""

    hardware_key, shape_key = _keys(hardware, shape)
    for entry in _matching_entries(hardware=hardware_key, path=path):
        if isinstance(entry.get("shape"), dict) and ShapeFingerprint.from_dict(entry["shape"]) == shape_key:
            return ConfigSpec.from_dict(entry["config"])
    return None


def iter_deployed_configs(
    *,
    hardware: EnvironmentFingerprint | dict[str, Any],
    path: str | Path = DEFAULT_DEPLOYED_CONFIGS_PATH,
) -> tuple[tuple[ShapeFingerprint, ConfigSpec], ...]:
    """Every exact-environment deployment as (shape, config) pairs."""

    hardware_key = (
        hardware if isinstance(hardware, EnvironmentFingerprint) else EnvironmentFingerprint.from_dict(hardware)
    )
    pairs = []
    for entry in _matching_entries(hardware=hardware_key, path=path):
        if isinstance(entry.get("shape"), dict) and isinstance(entry.get("config"), dict):
            pairs.append((ShapeFingerprint.from_dict(entry["shape"]), ConfigSpec.from_dict(entry["config"])))
    return tuple(pairs)


def publish_deployed_config(
    *,
    hardware: EnvironmentFingerprint | dict[str, Any],
    shape: ShapeFingerprint | dict[str, Any],
    config: ConfigSpec,
    path: str | Path = DEFAULT_DEPLOYED_CONFIGS_PATH,
) -> Path:
    """Replace (or add) one exact winner in the deployment table."""

    hardware_key, shape_key = _keys(hardware, shape)
    target = Path(path)
    try:
        document = _load(target)
    except FileNotFoundError:
        document = {"schema_version": DEPLOYMENT_SCHEMA_VERSION, "bundles": []}
    if document.get("schema_version") != DEPLOYMENT_SCHEMA_VERSION:
        document = {"schema_version": DEPLOYMENT_SCHEMA_VERSION, "bundles": []}
    bundle: dict[str, Any] | None = None
    for candidate in document["bundles"]:
        if (
            isinstance(candidate, dict)
            and isinstance(candidate.get("hardware"), dict)
            and EnvironmentFingerprint.from_dict(candidate["hardware"]).measurement_identity
            == hardware_key.measurement_identity
        ):
            bundle = candidate
            break
    if bundle is None:
        bundle = {"hardware": hardware_key.to_dict(), "entries": []}
        document["bundles"].append(bundle)
    else:
        bundle["hardware"] = hardware_key.to_dict()
    entries = bundle.setdefault("entries", [])
    replacement = {"shape": shape_key.to_dict(), "config": config.to_dict()}
    for index, entry in enumerate(entries):
        if isinstance(entry, dict) and isinstance(entry.get("shape"), dict) and ShapeFingerprint.from_dict(entry["shape"]) == shape_key:
            entries[index] = replacement
            break
    else:
        entries.append(replacement)
    target.parent.mkdir(parents=True, exist_ok=True)
    target.write_text(json.dumps(document, ensure_ascii=False, indent=2, allow_nan=False) + "\n", encoding="utf-8")
    return target


__all__ = [
    "DEFAULT_DEPLOYED_CONFIGS_PATH",
    "DEPLOYMENT_SCHEMA_VERSION",
    "EnvironmentFingerprint",
    "ShapeFingerprint",
    "iter_deployed_configs",
    "publish_deployed_config",
    "resolve_deployed_config",
]
