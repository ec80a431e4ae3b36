"""Build execution plans from typed search configurations.

Mirrors the reference's static compiler (``solution/plan_builder.py``):
``ConstraintViolation`` (:52-65), ``CompileRejection`` (:68-83),
``ConfigRejectedError`` (:86-94), ``CompilationResult`` (:97-121),
``HardwareCapabilities.detect`` (:124-200) and ``PlanBuilder.evaluate/build``
(:206-263).  A config either compiles to exactly one ``ExecutionPlan`` or is
rejected with structured violations; nothing is substituted.  The rules are
the sm_100a kernels' real constraints: a compute capability 10.0 device with
libb200tx loaded, inference only, head_dim 64, 16-byte row pitches, and the
schedule rules of the reference runtimes (:294-350,
solution/shape14/planning.py:13-41).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import torch

from . import _native
from .config import (
    AttentionBackend,
    ConfigSpec,
    FFNBackend,
    PrecisionPlan,
    ResidualNormBackend,
    RuntimeBackend,
    fp32_update_roles,
)
from .plan import ExecutionContext, ExecutionPlan, ExpectedExecutionTrace

Reject = Callable[[str, str, str], None]

SUPPORTED_HEAD_DIMS = frozenset({64})
# Head dims built into the CUDA-core attention (b200tx_attention_generic).
SIMT_HEAD_DIMS = frozenset({8, 16, 32, 64, 128, 256})
MMA_HEAD_DIMS = frozenset({8, 16, 32, 64, 128})
# d_model of the fused boundaries: the MLP form holds a row in one warp's
# registers; the Linear form also runs as a row-complete tcgen05 GEMM.
BOUNDARY_WIDTHS = frozenset({32, 64, 128})
LINEAR_BOUNDARY_WIDTHS = BOUNDARY_WIDTHS | {512, 768, 1024}
# The attention variants that read a key padding mask (B200TX_ATTN_QUAD,
# B200TX_ATTN_PERSISTENT, B200TX_ATTN_DUO and B200TX_ATTN_PINGPONG).
SM100_QUAD_ATTENTION_VARIANT = 2
SM100_MASKED_ATTENTION_VARIANTS = frozenset({2, 3, 4, 5})
SUPPORTED_IO_DTYPES = frozenset({torch.float32, torch.bfloat16})
_INT32_MAX = 2**31 - 1


@dataclass(frozen=True, slots=True)
class ConstraintViolation:
    """One statically known reason a configuration cannot execute."""

    code: str
    field: str
    message: str

    def to_dict(self) -> dict[str, str]:
        return {"code": self.code, "field": self.field, "message": self.message}


@dataclass(frozen=True, slots=True)
class CompileRejection:
    """Structured rejection retained as an infeasible search observation."""

    config_id: str
    violations: tuple[ConstraintViolation, ...]

    def __post_init__(self) -> None:
        if not self.violations:
            raise ValueError("CompileRejection requires at least one violation")

    def to_dict(self) -> dict[str, Any]:
        return {
            "config_id": self.config_id,
            "violations": [violation.to_dict() for violation in self.violations],
        }


class ConfigRejectedError(ValueError):
    """Raised when strict compilation receives a configuration it cannot run."""

    def __init__(self, rejection: CompileRejection) -> None:
        self.rejection = rejection
        summary = "; ".join(f"{item.field}:{item.code}" for item in rejection.violations)
        super().__init__(f"configuration {rejection.config_id} rejected: {summary}")


@dataclass(frozen=True, slots=True)
class CompilationResult:
    """Non-throwing compiler result used by a search engine."""

    config_id: str
    plan: ExecutionPlan | None
    rejection: CompileRejection | None

    def __post_init__(self) -> None:
        if (self.plan is None) == (self.rejection is None):
            raise ValueError("exactly one of plan and rejection must be present")

    @property
    def accepted(self) -> bool:
        return self.plan is not None

    @property
    def violations(self) -> tuple[ConstraintViolation, ...]:
        return () if self.rejection is None else self.rejection.violations

    def require_plan(self) -> ExecutionPlan:
        if self.plan is not None:
            return self.plan
        assert self.rejection is not None
        raise ConfigRejectedError(self.rejection)


@dataclass(frozen=True, slots=True)
class HardwareCapabilities:
    """Injectable hardware/library snapshot used by static compilation."""

    device_type: str
    compute_capability: tuple[int, int] | None
    shared_memory_per_block: int | None
    sm_count: int | None
    kernel_library: bool

    @classmethod
    def detect(cls, device: torch.device) -> HardwareCapabilities:
        device_type = device.type
        capability: tuple[int, int] | None = None
        shared_memory: int | None = None
        sm_count: int | None = None
        if device_type == "cuda" and torch.cuda.is_available():
            index = device.index if device.index is not None else torch.cuda.current_device()
            capability = tuple(torch.cuda.get_device_capability(index))  # type: ignore[assignment]
            properties = torch.cuda.get_device_properties(index)
            shared_memory = int(
                getattr(
                    properties,
                    "shared_memory_per_block_optin",
                    properties.shared_memory_per_block,
                )
            )
            sm_count = int(properties.multi_processor_count)
        return cls(
            device_type=device_type,
            compute_capability=capability,
            shared_memory_per_block=shared_memory,
            sm_count=sm_count,
            kernel_library=_native.library_available(),
        )

    @classmethod
    def sm100(cls) -> HardwareCapabilities:
        """A B200 snapshot, for planning on a host without the GPU."""

        return cls(
            device_type="cuda",
            compute_capability=(10, 0),
            shared_memory_per_block=232448,
            sm_count=148,
            kernel_library=True,
        )

    @property
    def is_sm100(self) -> bool:
        return self.device_type == "cuda" and self.compute_capability == (10, 0)


class PlanBuilder:
    """Build exactly one execution plan without policy lookup or fallback."""

    def evaluate(
        self,
        config: ConfigSpec,
        context: ExecutionContext,
        hardware: HardwareCapabilities | None = None,
    ) -> CompilationResult:
        if not isinstance(config, ConfigSpec):
            raise TypeError("config must be ConfigSpec")
        if not isinstance(context, ExecutionContext):
            raise TypeError("context must be ExecutionContext")
        capabilities = hardware or HardwareCapabilities.detect(context.device)
        violations: list[ConstraintViolation] = []

        def reject(code: str, field: str, message: str) -> None:
            violations.append(ConstraintViolation(code, field, message))

        self._validate_context(context, capabilities, reject)
        inner_context = self._validate_runtime(config, context, reject)
        self._validate_shapes(config, inner_context, reject)

        if violations:
            rejection = CompileRejection(config.config_id, tuple(violations))
            return CompilationResult(config.config_id, None, rejection)
        plan = self._build_plan(config, context, inner_context)
        return CompilationResult(config.config_id, plan, None)

    def build(
        self,
        config: ConfigSpec,
        context: ExecutionContext,
        hardware: HardwareCapabilities | None = None,
    ) -> ExecutionPlan:
        """Build a plan or raise ConfigRejectedError; never substitute a config."""

        return self.evaluate(config, context, hardware).require_plan()

    @staticmethod
    def _validate_context(
        context: ExecutionContext, hardware: HardwareCapabilities, reject: Reject
    ) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads"):
            value = getattr(context, name)
            if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
                reject("non_positive", name, f"{name} must be positive")
        if context.num_heads > 0 and context.d_model % context.num_heads:
            reject("not_divisible", "num_heads", "d_model must be divisible by num_heads")
        if context.has_valid_token_mask and not context.mask_compatible:
            reject(
                "incompatible_mask",
                "valid_token_mask",
                "token mask does not match the input shape, device, or dtype",
            )
        if hardware.device_type != context.device.type:
            reject(
                "device_mismatch",
                "hardware.device_type",
                "hardware capabilities do not describe the input device",
            )
        if context.device.type != "cuda":
            reject("requires_cuda", "device", "the sm100 kernels run on CUDA devices only")
        elif not hardware.is_sm100:
            reject(
                "requires_sm100",
                "hardware.compute_capability",
                f"libb200tx is built for sm_100a; device reports {hardware.compute_capability}",
            )
        if not hardware.kernel_library:
            reject("backend_unavailable", "kernel_library", "libb200tx.so is not loadable")
        if not context.inference:
            reject(
                "requires_inference",
                "context",
                "the sm100 kernels implement inference only (no autograd)",
            )
        if context.dtype not in SUPPORTED_IO_DTYPES:
            reject(
                "unsupported_dtype",
                "dtype",
                f"input dtype {context.dtype_name} is not float32 or bfloat16",
            )
        if not context.input_contiguous:
            reject("requires_contiguous_input", "input", "input must be contiguous")

    @staticmethod
    def _validate_runtime(
        config: ConfigSpec, context: ExecutionContext, reject: Reject
    ) -> ExecutionContext:
        runtime = config.schedule.runtime
        if runtime in (RuntimeBackend.EAGER, RuntimeBackend.CUDA_GRAPH):
            return context
        if runtime is RuntimeBackend.BATCH_TILED_CUDA_GRAPH:
            tile = config.schedule.batch_tile_size
            assert tile is not None
            if tile >= context.batch_size:
                reject(
                    "tile_not_smaller_than_batch",
                    "schedule.batch_tile_size",
                    "batch tile must be smaller than the logical batch",
                )
            return context.with_batch_size(tile)
        if runtime is RuntimeBackend.STREAMED:
            from .shape14.planning import validate_streamed_runtime

            return validate_streamed_runtime(config, context, reject)
        if runtime is RuntimeBackend.SEQUENCE_RESIDENT:
            from .runtimes.sequence_resident import sequence_resident_supported

            why = sequence_resident_supported(
                d_model=context.d_model,
                ffn_dim=context.ffn_dim if context.ffn_dim is not None else -1,
                num_heads=context.num_heads,
                seq_len=context.seq_len,
                num_layers=context.num_layers if context.num_layers is not None else 0,
                causal=bool(context.causal),
            )
            if why is not None:
                reject("unsupported_shape", "schedule.runtime", f"the whole-forward kernel is {why}")
            if context.has_valid_token_mask:
                reject("mask_not_supported", "schedule.runtime", "the whole-forward kernel takes no padding mask")
            if context.dtype != torch.float32:
                reject("unsupported_dtype", "schedule.runtime", "the whole-forward kernel takes float32 input")
            return context
        raise AssertionError(f"unhandled runtime backend: {runtime}")

    @staticmethod
    def _validate_shapes(config: ConfigSpec, context: ExecutionContext, reject: Reject) -> None:
        head_dim = context.head_dim
        launch = config.schedule.attention_launch
        if (
            context.has_valid_token_mask
            and config.program.attention is AttentionBackend.SM100_FLASH
            and launch is not None
            and launch.kernel_variant not in SM100_MASKED_ATTENTION_VARIANTS
        ):
            reject(
                "mask_not_supported",
                "schedule.attention_launch",
                "padding masks are built into the quad (block_m 512, block_n 64, kv_stages 6), "
                "persistent (256, 64, 8), duo (256, 64, 4) and pingpong (256, 128, 4) attention "
                "variants only",
            )
        if config.program.attention is AttentionBackend.SM100_FLASH:
            if head_dim is not None and head_dim not in SUPPORTED_HEAD_DIMS:
                reject(
                    "unsupported_shape",
                    "program.attention",
                    f"sm100 flash attention is built for head_dim 64, not {head_dim}",
                )
        elif config.program.attention is AttentionBackend.SM100_SIMT:
            if head_dim is not None and head_dim not in SIMT_HEAD_DIMS:
                reject(
                    "unsupported_shape",
                    "program.attention",
                    f"sm100 CUDA-core attention is built for head_dim {sorted(SIMT_HEAD_DIMS)}, not {head_dim}",
                )
        elif config.program.attention is AttentionBackend.SM100_MMA:
            if head_dim is not None and head_dim not in MMA_HEAD_DIMS:
                reject(
                    "unsupported_shape",
                    "program.attention",
                    f"sm100 warp-MMA attention is built for head_dim {sorted(MMA_HEAD_DIMS)}, not {head_dim}",
                )
        if context.d_model % 8:
            reject(
                "unsupported_shape",
                "d_model",
                "d_model must be a multiple of 8 (16-byte TMA row pitch)",
            )
        ffn_dim = context.ffn_dim
        if ffn_dim is None or ffn_dim <= 0:
            reject("non_positive", "ffn_dim", "ffn_dim must be positive")
        elif ffn_dim % 8:
            reject(
                "unsupported_shape",
                "ffn_dim",
                "ffn_dim must be a multiple of 8 (16-byte TMA row pitch)",
            )
        # Fused block boundaries (reference rules: solution/plan_builder.py:669-697,
        # 783-805): a whole row of d_model in a warp's registers.
        program = config.program
        if program.residual_norm is ResidualNormBackend.SM100_LINEAR_MIXED:
            if context.d_model not in LINEAR_BOUNDARY_WIDTHS:
                reject(
                    "unsupported_shape",
                    "program.residual_norm",
                    f"the fused Linear residual-norm boundary is built for d_model {sorted(LINEAR_BOUNDARY_WIDTHS)}, "
                    f"not {context.d_model}",
                )
        if program.ffn is FFNBackend.SM100_FUSED_MLP_BOUNDARY:
            if program.residual_norm is not ResidualNormBackend.SM100_LINEAR_MIXED:
                reject(
                    "backend_incompatible",
                    "program.residual_norm",
                    "the fused MLP boundary requires the fused Linear residual-norm boundary",
                )
            if context.d_model not in BOUNDARY_WIDTHS:
                reject(
                    "unsupported_shape",
                    "program.ffn",
                    f"the fused MLP boundary is built for d_model {sorted(BOUNDARY_WIDTHS)}, not {context.d_model}",
                )
            if ffn_dim is not None and ffn_dim > 0 and ffn_dim % 16:
                reject(
                    "unsupported_shape",
                    "ffn_dim",
                    "the fused MLP boundary gives each warp 16 hidden columns at a time: ffn_dim % 16 == 0",
                )
        if context.num_layers is None or context.num_layers <= 0:
            reject("non_positive", "num_layers", "num_layers must be positive")
        tokens = context.batch_size * context.seq_len
        if tokens > _INT32_MAX:
            reject(
                "unsupported_shape",
                "batch_size",
                "one launch handles at most 2^31-1 token rows; use the streamed runtime",
            )
        if head_dim:
            q_tiles = (context.seq_len + 127) // 128
            if q_tiles * context.num_heads * context.batch_size > _INT32_MAX:
                reject(
                    "unsupported_shape",
                    "seq_len",
                    "attention grid exceeds one launch; use the streamed runtime",
                )

    @staticmethod
    def _build_plan(
        config: ConfigSpec, outer: ExecutionContext, inner: ExecutionContext
    ) -> ExecutionPlan:
        program = config.program
        schedule = config.schedule
        fp32_roles = fp32_update_roles(program.precision_plan)
        out_update = "float32" if "attention_output_projection" in fp32_roles else "bfloat16"
        ffn_update = "float32" if "ffn_output_projection" in fp32_roles else "bfloat16"
        layers = max(0, int(inner.num_layers or 0))
        expected = ExpectedExecutionTrace(
            runtime_backend=schedule.runtime,
            attention_backend=program.attention,
            qkv_projection_backend=program.qkv_projection,
            attention_output_projection_backend=program.attention_output_projection,
            ffn_input_projection_backend=program.ffn_input_projection,
            ffn_output_projection_backend=program.ffn_output_projection,
            precision_plan=program.precision_plan,
            qkv_materialization=program.qkv_materialization,
            attention_output_bridge=program.attention_output_bridge,
            attention_output_layout=config.attention_output_layout,
            ffn_backend=program.ffn,
            residual_norm_backend=program.residual_norm,
            initial_norm_backend=program.initial_norm,
            attention_compute_dtype="bfloat16",
            qkv_projection_compute_dtype="bfloat16",
            attention_output_projection_compute_dtype="bfloat16",
            ffn_input_projection_compute_dtype="bfloat16",
            ffn_activation_output_dtype="bfloat16",
            ffn_output_projection_compute_dtype="bfloat16",
            attention_calls=layers,
            qkv_projection_calls=layers,
            attention_output_projection_calls=layers,
            ffn_calls=layers,
            ffn_input_projection_calls=layers,
            ffn_output_projection_calls=layers,
            residual_norm_calls=2 * layers,
            initial_norm_calls=1 if layers else 0,
            runtime_calls=1,
            attention_launch=schedule.attention_launch,
            qkv_launch=schedule.qkv_launch,
            attention_output_projection_launch=schedule.attention_output_projection_launch,
            residual_norm_launch=schedule.residual_norm_launch,
            initial_norm_launch=schedule.initial_norm_launch,
            ffn_launch=schedule.ffn_launch,
            ffn_input_launch=schedule.ffn_input_launch,
        )
        return ExecutionPlan(
            config=config,
            outer_context=outer,
            inner_context=inner,
            attention_backend=program.attention,
            attention_compute_dtype="bfloat16",
            qkv_projection_backend=program.qkv_projection,
            qkv_projection_compute_dtype="bfloat16",
            qkv_materialization=program.qkv_materialization,
            attention_output_bridge=program.attention_output_bridge,
            attention_output_layout=config.attention_output_layout,
            attention_output_projection_backend=program.attention_output_projection,
            attention_output_projection_compute_dtype="bfloat16",
            attention_output_update_dtype=out_update,
            ffn_backend=program.ffn,
            ffn_input_projection_backend=program.ffn_input_projection,
            ffn_input_projection_compute_dtype="bfloat16",
            ffn_activation_output_dtype="bfloat16",
            ffn_output_projection_backend=program.ffn_output_projection,
            ffn_output_projection_compute_dtype="bfloat16",
            ffn_output_update_dtype=ffn_update,
            precision_plan=program.precision_plan,
            residual_norm_backend=program.residual_norm,
            initial_norm_backend=program.initial_norm,
            runtime_backend=schedule.runtime,
            batch_tile_size=schedule.batch_tile_size,
            microbatch_size=schedule.microbatch_size,
            reuse_unchanged_input=schedule.reuse_unchanged_input,
            attention_launch=schedule.attention_launch,
            qkv_launch=schedule.qkv_launch,
            attention_output_projection_launch=schedule.attention_output_projection_launch,
            residual_norm_launch=schedule.residual_norm_launch,
            initial_norm_launch=schedule.initial_norm_launch,
            ffn_launch=schedule.ffn_launch,
            ffn_input_launch=schedule.ffn_input_launch,
            output_dtype=outer.dtype_name,
            expected_trace=expected,
        )


__all__ = [
    "CompilationResult",
    "CompileRejection",
    "ConfigRejectedError",
    "ConstraintViolation",
    "HardwareCapabilities",
    "PlanBuilder",
    "PrecisionPlan",
]
