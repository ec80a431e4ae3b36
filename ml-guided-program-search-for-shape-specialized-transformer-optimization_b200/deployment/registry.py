"""Deployed programs per (measured environment, workload shape).

The interface is the reference's deployment registry (deployment/registry.py:
``ShapeFingerprint`` :20-60, ``resolve_deployed_config`` :107-121,
``iter_deployed_configs`` :124-148, ``publish_deployed_config`` :151-205) and
its JSON document, so a table written by either loads in the other's schema:

    {"schema_version": 4,
     "bundles": [{"hardware": <EnvironmentFingerprint.to_dict()>,
                  "entries": [{"shape": <ShapeFingerprint.to_dict()>,
                               "config": <ConfigSpec.to_dict()>}, ...]}, ...]}

Lookups are exact on both keys (the environment by its measurement identity,
which leaves out the source digest); a miss returns ``None`` and the model
runs its default program.

This implementation keeps a parsed index of each table file, rebuilt only
when the file's size or modification time changes, so resolving a config on
a model's first call is a dictionary lookup, not a JSON parse; and it
publishes through a temporary file and an atomic rename, so a reader never
sees a half-written table.
"""

from __future__ import annotations

import json
import os
import tempfile
import threading
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Any

from solution.config import ConfigSpec

from .environment import EnvironmentFingerprint

DEFAULT_DEPLOYED_CONFIGS_PATH = Path(__file__).resolve().parent / "deployed_configs.json"
DEPLOYMENT_SCHEMA_VERSION = 4


@dataclass(frozen=True, slots=True)
class ShapeFingerprint:
    """The workload a deployed program was measured on (every field must match)."""

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
        # Each field is read through its own annotated type (a missing key
        # raises KeyError, as any malformed entry should).
        casts = {"int": int, "bool": bool, "str": str, "float": float}
        return cls(**{f.name: casts[str(f.type)](value[f.name]) for f in fields(cls)})

    def to_dict(self) -> dict[str, Any]:
        return {f.name: getattr(self, f.name) for f in fields(self)}


def _environment(value: EnvironmentFingerprint | dict[str, Any]) -> EnvironmentFingerprint:
    return value if isinstance(value, EnvironmentFingerprint) else EnvironmentFingerprint.from_dict(value)


def _shape(value: ShapeFingerprint | dict[str, Any]) -> ShapeFingerprint:
    return value if isinstance(value, ShapeFingerprint) else ShapeFingerprint.from_dict(value)


class _TableIndex:
    """One table file parsed into {measurement identity: {shape: config dict}}.

    The first bundle of an identity and the first entry of a shape win, as in
    a linear scan of the document.  Malformed bundles and entries are left out.
    """

    def __init__(self, document: dict[str, Any] | None) -> None:
        self.by_identity: dict[str, dict[ShapeFingerprint, dict[str, Any]]] = {}
        if document is None or document.get("schema_version") != DEPLOYMENT_SCHEMA_VERSION:
            return
        for bundle in document.get("bundles", []):
            if not isinstance(bundle, dict) or not isinstance(bundle.get("hardware"), dict):
                continue
            identity = EnvironmentFingerprint.from_dict(bundle["hardware"]).measurement_identity
            if identity in self.by_identity:
                continue
            shapes: dict[ShapeFingerprint, dict[str, Any]] = {}
            for entry in bundle.get("entries", []):
                if not isinstance(entry, dict):
                    continue
                if isinstance(entry.get("shape"), dict) and isinstance(entry.get("config"), dict):
                    shapes.setdefault(ShapeFingerprint.from_dict(entry["shape"]), entry["config"])
            self.by_identity[identity] = shapes


_index_lock = threading.Lock()
_index_cache: dict[Path, tuple[tuple[int, int], _TableIndex]] = {}


def _read_document(path: Path) -> dict[str, Any]:
    value = json.loads(path.read_text(encoding="utf-8"))
    if not isinstance(value, dict) or not isinstance(value.get("bundles"), list):
        raise ValueError("deployed config file must contain a bundles array")
    return value


def _index(path: str | Path) -> _TableIndex:
    """The parsed index of ``path`` (empty when the file does not exist)."""

    target = Path(path).resolve()
    try:
        stat = target.stat()
    except FileNotFoundError:
        return _TableIndex(None)
    stamp = (stat.st_mtime_ns, stat.st_size)
    with _index_lock:
        cached = _index_cache.get(target)
        if cached is not None and cached[0] == stamp:
            return cached[1]
    index = _TableIndex(_read_document(target))
    with _index_lock:
        _index_cache[target] = (stamp, index)
    return index


def resolve_deployed_config(
    *,
    hardware: EnvironmentFingerprint | dict[str, Any],
    shape: ShapeFingerprint | dict[str, Any],
    path: str | Path = DEFAULT_DEPLOYED_CONFIGS_PATH,
) -> ConfigSpec | None:
    """The program deployed for exactly this environment and shape, else ``None``."""

    shapes = _index(path).by_identity.get(_environment(hardware).measurement_identity, {})
    config = shapes.get(_shape(shape))
    return None if config is None else ConfigSpec.from_dict(config)


def iter_deployed_configs(
    *,
    hardware: EnvironmentFingerprint | dict[str, Any],
    path: str | Path = DEFAULT_DEPLOYED_CONFIGS_PATH,
) -> tuple[tuple[ShapeFingerprint, ConfigSpec], ...]:
    """Every (shape, config) deployed for this environment, in table order."""

    shapes = _index(path).by_identity.get(_environment(hardware).measurement_identity, {})
    return tuple((shape, ConfigSpec.from_dict(config)) for shape, config in shapes.items())


def publish_deployed_config(
    *,
    hardware: EnvironmentFingerprint | dict[str, Any],
    shape: ShapeFingerprint | dict[str, Any],
    config: ConfigSpec,
    path: str | Path = DEFAULT_DEPLOYED_CONFIGS_PATH,
) -> Path:
    """Record ``config`` as the program for this environment and shape.

    The environment's bundle (matched by measurement identity) takes the new
    hardware record and the entry, replacing one of the same shape; a table
    of another schema version is started afresh.  Written atomically.
    """

    environment = _environment(hardware)
    key = _shape(shape)
    target = Path(path)
    try:
        document = _read_document(target)
    except FileNotFoundError:
        document = None
    if document is None or document.get("schema_version") != DEPLOYMENT_SCHEMA_VERSION:
        document = {"schema_version": DEPLOYMENT_SCHEMA_VERSION, "bundles": []}
    identity = environment.measurement_identity
    bundle = next(
        (
            b
            for b in document["bundles"]
            if isinstance(b, dict)
            and isinstance(b.get("hardware"), dict)
            and EnvironmentFingerprint.from_dict(b["hardware"]).measurement_identity == identity
        ),
        None,
    )
    if bundle is None:
        bundle = {"hardware": None, "entries": []}
        document["bundles"].append(bundle)
    bundle["hardware"] = environment.to_dict()
    record = {"shape": key.to_dict(), "config": config.to_dict()}
    entries = [
        e
        for e in bundle.get("entries", [])
        if not (isinstance(e, dict) and isinstance(e.get("shape"), dict) and ShapeFingerprint.from_dict(e["shape"]) == key)
    ]
    # The replaced entry keeps its position; a new shape goes last.
    position = next(
        (
            i
            for i, e in enumerate(bundle.get("entries", []))
            if isinstance(e, dict) and isinstance(e.get("shape"), dict) and ShapeFingerprint.from_dict(e["shape"]) == key
        ),
        len(entries),
    )
    entries.insert(position, record)
    bundle["entries"] = entries

    target.parent.mkdir(parents=True, exist_ok=True)
    text = json.dumps(document, ensure_ascii=False, indent=2, allow_nan=False) + "\n"
    handle, temporary = tempfile.mkstemp(prefix=target.name + ".", suffix=".tmp", dir=target.parent)
    try:
        with os.fdopen(handle, "w", encoding="utf-8") as stream:
            stream.write(text)
        os.replace(temporary, target)
    except BaseException:
        Path(temporary).unlink(missing_ok=True)
        raise
    with _index_lock:
        _index_cache.pop(target.resolve(), None)
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
