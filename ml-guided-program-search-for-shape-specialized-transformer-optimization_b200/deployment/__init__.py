"""Deployed configuration registry (reference: deployment/__init__.py)."""

from .registry import (
    DEFAULT_DEPLOYED_CONFIGS_PATH,
    DEPLOYMENT_SCHEMA_VERSION,
    EnvironmentFingerprint,
    ShapeFingerprint,
    iter_deployed_configs,
    publish_deployed_config,
    resolve_deployed_config,
)

__all__ = [
    "DEFAULT_DEPLOYED_CONFIGS_PATH",
    "DEPLOYMENT_SCHEMA_VERSION",
    "EnvironmentFingerprint",
    "ShapeFingerprint",
    "iter_deployed_configs",
    "publish_deployed_config",
    "resolve_deployed_config",
]
