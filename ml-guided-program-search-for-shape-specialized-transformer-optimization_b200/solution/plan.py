"""Immutable execution plans built from typed Transformer configurations.

Mirrors the reference's ``solution/plan.py``: ``ExecutionContext`` (:30-66),
``ExpectedExecutionTrace`` (:69-185) and ``ExecutionPlan`` (:188-341).  The
plan is the single object ``UserOptimizedTransformer.forward`` executes; the
expected trace derived from it is compared against the markers the kernels
report at run time, so a drift between plan and execution raises instead of
passing silently.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any

import torch

from .config import (
    AttentionBackend,
    AttentionOutputBridge,
    AttentionOutputLayout,
    ConfigSpec,
    FFNBackend,
    InitialNormBackend,
    PrecisionPlan,
    ProjectionBackend,
    QKVMaterialization,
    ResidualNormBackend,
    RuntimeBackend,
    Sm100AttentionParams,
    Sm100GemmParams,
    Sm100NormParams,
)


@dataclass(frozen=True, slots=True)
class ExecutionContext:
    """Input and model facts that affect plan eligibility (reference plan.py:30-66)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    causal: bool
    device: torch.device
    dtype: torch.dtype
    training: bool
    grad_enabled: bool
    input_contiguous: bool
    has_valid_token_mask: bool
    mask_compatible: bool
    ffn_dim: int | None = None
    num_layers: int | None = None

    @property
    def head_dim(self) -> int | None:
        if self.num_heads <= 0 or self.d_model % self.num_heads:
            return None
        return self.d_model // self.num_heads

    @property
    def dtype_name(self) -> str:
        return str(self.dtype).removeprefix("torch.")

    @property
    def inference(self) -> bool:
        return not self.training and not self.grad_enabled

    @property
    def tokens(self) -> int:
        return self.batch_size * self.seq_len

    def with_batch_size(self, batch_size: int) -> ExecutionContext:
        """The inner context seen by a batch-tiled or streamed schedule."""

        return replace(self, batch_size=batch_size)


@dataclass(frozen=True, slots=True)
class ExpectedExecutionTrace:
    """Path evidence derived from the plan (reference plan.py:69-185)."""

    runtime_backend: RuntimeBackend
    attention_backend: AttentionBackend
    qkv_projection_backend: ProjectionBackend
    attention_output_projection_backend: ProjectionBackend
    ffn_input_projection_backend: ProjectionBackend
    ffn_output_projection_backend: ProjectionBackend
    precision_plan: PrecisionPlan
    qkv_materialization: QKVMaterialization
    attention_output_bridge: AttentionOutputBridge
    attention_output_layout: AttentionOutputLayout
    ffn_backend: FFNBackend
    residual_norm_backend: ResidualNormBackend
    initial_norm_backend: InitialNormBackend
    attention_compute_dtype: str
    qkv_projection_compute_dtype: str
    attention_output_projection_compute_dtype: str
    ffn_input_projection_compute_dtype: str
    ffn_activation_output_dtype: str
    ffn_output_projection_compute_dtype: str
    attention_calls: int
    qkv_projection_calls: int
    attention_output_projection_calls: int
    ffn_calls: int
    ffn_input_projection_calls: int
    ffn_output_projection_calls: int
    residual_norm_calls: int
    initial_norm_calls: int
    runtime_calls: int
    attention_launch: Sm100AttentionParams | None = None
    qkv_launch: Sm100GemmParams | None = None
    attention_output_projection_launch: Sm100GemmParams | None = None
    residual_norm_launch: Sm100NormParams | None = None
    initial_norm_launch: Sm100NormParams | None = None
    ffn_launch: Sm100GemmParams | None = None
    ffn_input_launch: Sm100GemmParams | None = None

    def to_dict(self) -> dict[str, Any]:
        def dump(value: Any) -> Any:
            return None if value is None else value.to_dict()

        return {
            "runtime_backend": self.runtime_backend.value,
            "attention_backend": self.attention_backend.value,
            "qkv_projection_backend": self.qkv_projection_backend.value,
            "attention_output_projection_backend": self.attention_output_projection_backend.value,
            "ffn_input_projection_backend": self.ffn_input_projection_backend.value,
            "ffn_output_projection_backend": self.ffn_output_projection_backend.value,
            "precision_plan": self.precision_plan.value,
            "qkv_materialization": self.qkv_materialization.value,
            "attention_output_bridge": self.attention_output_bridge.value,
            "attention_output_layout": self.attention_output_layout.value,
            "ffn_backend": self.ffn_backend.value,
            "residual_norm_backend": self.residual_norm_backend.value,
            "initial_norm_backend": self.initial_norm_backend.value,
            "attention_compute_dtype": self.attention_compute_dtype,
            "qkv_projection_compute_dtype": self.qkv_projection_compute_dtype,
            "attention_output_projection_compute_dtype": (
                self.attention_output_projection_compute_dtype
            ),
            "ffn_input_projection_compute_dtype": self.ffn_input_projection_compute_dtype,
            "ffn_activation_output_dtype": self.ffn_activation_output_dtype,
            "ffn_output_projection_compute_dtype": self.ffn_output_projection_compute_dtype,
            "attention_calls": self.attention_calls,
            "qkv_projection_calls": self.qkv_projection_calls,
            "attention_output_projection_calls": self.attention_output_projection_calls,
            "ffn_calls": self.ffn_calls,
            "ffn_input_projection_calls": self.ffn_input_projection_calls,
            "ffn_output_projection_calls": self.ffn_output_projection_calls,
            "residual_norm_calls": self.residual_norm_calls,
            "initial_norm_calls": self.initial_norm_calls,
            "runtime_calls": self.runtime_calls,
            "attention_launch": dump(self.attention_launch),
            "qkv_launch": dump(self.qkv_launch),
            "attention_output_projection_launch": dump(self.attention_output_projection_launch),
            "residual_norm_launch": dump(self.residual_norm_launch),
            "initial_norm_launch": dump(self.initial_norm_launch),
            "ffn_launch": dump(self.ffn_launch),
            "ffn_input_launch": dump(self.ffn_input_launch),
            "complete": True,
        }


@dataclass(frozen=True, slots=True)
class ExecutionPlan:
    """Strict plan that forward executes without hidden fallback (reference :188-341)."""

    config: ConfigSpec
    outer_context: ExecutionContext
    inner_context: ExecutionContext
    attention_backend: AttentionBackend
    attention_compute_dtype: str
    qkv_projection_backend: ProjectionBackend
    qkv_projection_compute_dtype: str
    qkv_materialization: QKVMaterialization
    attention_output_bridge: AttentionOutputBridge
    attention_output_layout: AttentionOutputLayout
    attention_output_projection_backend: ProjectionBackend
    attention_output_projection_compute_dtype: str
    attention_output_update_dtype: str
    ffn_backend: FFNBackend
    ffn_input_projection_backend: ProjectionBackend
    ffn_input_projection_compute_dtype: str
    ffn_activation_output_dtype: str
    ffn_output_projection_backend: ProjectionBackend
    ffn_output_projection_compute_dtype: str
    ffn_output_update_dtype: str
    precision_plan: PrecisionPlan
    residual_norm_backend: ResidualNormBackend
    initial_norm_backend: InitialNormBackend
    runtime_backend: RuntimeBackend
    batch_tile_size: int | None
    microbatch_size: int | None
    reuse_unchanged_input: bool
    attention_launch: Sm100AttentionParams | None
    qkv_launch: Sm100GemmParams | None
    attention_output_projection_launch: Sm100GemmParams | None
    residual_norm_launch: Sm100NormParams | None
    initial_norm_launch: Sm100NormParams | None
    ffn_launch: Sm100GemmParams | None
    ffn_input_launch: Sm100GemmParams | None
    output_dtype: str
    expected_trace: ExpectedExecutionTrace

    @property
    def config_id(self) -> str:
        return self.config.config_id

    @property
    def use_cuda_graph(self) -> bool:
        return self.runtime_backend is RuntimeBackend.CUDA_GRAPH

    @property
    def use_batch_tiled_cuda_graph(self) -> bool:
        return self.runtime_backend is RuntimeBackend.BATCH_TILED_CUDA_GRAPH

    @property
    def use_streamed_execution(self) -> bool:
        return self.runtime_backend is RuntimeBackend.STREAMED

    @property
    def use_sequence_resident(self) -> bool:
        return self.runtime_backend is RuntimeBackend.SEQUENCE_RESIDENT

    def describe(self) -> dict[str, Any]:
        """Serialise the plan and its derived evidence (reference plan.py:266-341)."""

        def dump(value: Any) -> Any:
            return None if value is None else value.to_dict()

        return {
            "config": self.config.to_dict(),
            "qkv_projection": "packed",
            "qkv_projection_backend": self.qkv_projection_backend.value,
            "qkv_projection_compute_dtype": self.qkv_projection_compute_dtype,
            "qkv_materialization": self.qkv_materialization.value,
            "attention_backend": self.attention_backend.value,
            "attention_compute_dtype": self.attention_compute_dtype,
            "attention_output_bridge": self.attention_output_bridge.value,
            "attention_output_layout": self.attention_output_layout.value,
            "attention_output_projection_backend": self.attention_output_projection_backend.value,
            "attention_output_projection_compute_dtype": (
                self.attention_output_projection_compute_dtype
            ),
            "attention_output_update_dtype": self.attention_output_update_dtype,
            "ffn_backend": self.ffn_backend.value,
            "ffn_input_projection_backend": self.ffn_input_projection_backend.value,
            "ffn_input_projection_compute_dtype": self.ffn_input_projection_compute_dtype,
            "ffn_activation_output_dtype": self.ffn_activation_output_dtype,
            "ffn_output_projection_backend": self.ffn_output_projection_backend.value,
            "ffn_output_projection_compute_dtype": self.ffn_output_projection_compute_dtype,
            "ffn_output_update_dtype": self.ffn_output_update_dtype,
            "precision_plan": self.precision_plan.value,
            "residual_norm_backend": self.residual_norm_backend.value,
            "initial_norm_backend": self.initial_norm_backend.value,
            "runtime_backend": self.runtime_backend.value,
            "batch_tile_size": self.batch_tile_size,
            "microbatch_size": self.microbatch_size,
            "reuse_unchanged_input": self.reuse_unchanged_input,
            "attention_launch": dump(self.attention_launch),
            "qkv_launch": dump(self.qkv_launch),
            "attention_output_projection_launch": dump(self.attention_output_projection_launch),
            "residual_norm_launch": dump(self.residual_norm_launch),
            "initial_norm_launch": dump(self.initial_norm_launch),
            "ffn_launch": dump(self.ffn_launch),
            "ffn_input_launch": dump(self.ffn_input_launch),
            "output_dtype": self.output_dtype,
            "outer_batch_size": self.outer_context.batch_size,
            "inner_batch_size": self.inner_context.batch_size,
            "causal_mask": "online_causal" if self.outer_context.causal else "none",
            "valid_token_mask": (
                "direct_key_mask" if self.outer_context.has_valid_token_mask else "none"
            ),
        }


__all__ = ["ExecutionContext", "ExecutionPlan", "ExpectedExecutionTrace"]
