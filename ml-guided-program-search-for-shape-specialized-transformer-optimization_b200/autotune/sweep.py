"""Exhaustive timing sweep of a ``ProgramSearchSpace`` on the GPU.

The reference tunes with Optuna trials measured by its benchmarking harness
(autotune/optimization_loop.py, benchmarking/measurement_core.py:20-30: warm
up, then the median of CUDA-event timings).  The sm100 space is small enough
to measure exhaustively: every accepted config is installed on the model
(``configure_execution``), warmed up and timed with CUDA events (median of
``repeats``), and its output is checked against the portable program's output
on the same input before it may win.  ``publish_best`` writes the winner into
the deployment registry for this environment and shape, from where the model
resolves it on its next first call (reference deployment/registry.py flow).
"""

from __future__ import annotations

import statistics
from dataclasses import dataclass
from typing import Any

import torch

from solution.config import ConfigSpec, portable_config

from .search_space import ProgramSearchSpace


@dataclass(frozen=True)
class SweepResult:
    config: ConfigSpec
    median_ms: float
    max_abs_diff: float


def _time(model: Any, x: torch.Tensor, warmup: int, repeats: int) -> tuple[float, torch.Tensor]:
    with torch.inference_mode():
        for _ in range(warmup):
            y = model(x)
        torch.cuda.synchronize()
        times = []
        for _ in range(repeats):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            y = model(x)
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end))
    return statistics.median(times), y


def sweep(
    model: Any,
    x: torch.Tensor,
    space: ProgramSearchSpace,
    *,
    warmup: int = 3,
    repeats: int = 10,
    max_abs_tolerance: float = 2e-2,
    limit: int | None = None,
) -> list[SweepResult]:
    """Time every accepted config of `space` on `model(x)`; fastest first.

    Configs whose output differs from the portable program's by more than
    `max_abs_tolerance` are left out of the result.  `limit` caps the number
    of configs measured (in the space's enumeration order).
    """

    if x.device.type != "cuda":
        raise ValueError("the sweep measures on a CUDA input")
    model.configure_execution(config=portable_config())
    _, reference = _time(model, x, 1, 1)
    reference = reference.float().clone()
    results = []
    for count, config in enumerate(space.configs()):
        if limit is not None and count >= limit:
            break
        model.configure_execution(config=config)
        ms, y = _time(model, x, warmup, repeats)
        diff = float((y.float() - reference).abs().max())
        if diff <= max_abs_tolerance:
            results.append(SweepResult(config=config, median_ms=ms, max_abs_diff=diff))
    results.sort(key=lambda r: r.median_ms)
    return results


def publish_best(model: Any, x: torch.Tensor, results: list[SweepResult], *, path: Any = None) -> Any:
    """Publish the fastest result for this device and shape; returns the path."""

    if not results:
        raise ValueError("no sweep result to publish")
    from deployment.environment import ImplementationScope
    from deployment.registry import (
        DEFAULT_DEPLOYED_CONFIGS_PATH,
        EnvironmentFingerprint,
        ShapeFingerprint,
        publish_deployed_config,
    )
    from solution.shape14.defaults import is_streamed_shape

    batch, seq, d_model = x.shape
    scope = ImplementationScope.SHAPE14 if is_streamed_shape(seq, d_model) else ImplementationScope.RESIDENT
    cfg = model.config
    shape = ShapeFingerprint(
        batch_size=int(batch),
        qkv_dim=int(cfg.d_model),
        heads=int(cfg.num_heads),
        seq_len=int(seq),
        layers=int(cfg.num_layers),
        causal=bool(cfg.causal),
        ffn_dim=int(cfg.ffn_dim),
        dtype=str(x.dtype).removeprefix("torch."),
        padding_ratio=0.0,
        input_scale=1.0,
    )
    return publish_deployed_config(
        hardware=EnvironmentFingerprint.detect(x.device, scope=scope),
        shape=shape,
        config=results[0].config,
        path=DEFAULT_DEPLOYED_CONFIGS_PATH if path is None else path,
    )


__all__ = ["SweepResult", "publish_best", "sweep"]
