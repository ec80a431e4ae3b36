"""Typed, serialisable program space for the sm_100a Transformer forward.

Mirrors the reference's ``solution/config.py`` (schema v4, ``ConfigSpec`` at
:672-785, ``ProgramConfig`` :389-487, ``ScheduleConfig`` :490-669, canonical
JSON and ``config_id`` :760-775, ``portable_config`` :788-806): the same three
frozen dataclasses, the same exact-field JSON round trip, the same sha256
``config_id``, the same cross-field legality rules between a program choice and
the launch parameters it needs.  What changed is the vocabulary: every
mechanism value names an sm_100a kernel of libb200tx (or a schedule around
them), so the program search chooses among B200 kernel variants instead of
Triton/SDPA/torch.compile ones.  Schema version 5 marks that change; v4
documents are rejected rather than reinterpreted.
"""

from __future__ import annotations

import functools
import hashlib
import json
from dataclasses import dataclass, field
from enum import StrEnum
from typing import Any, ClassVar

CONFIG_SCHEMA_VERSION = 5


class AttentionBackend(StrEnum):
    """Attention primitives (reference values: solution/config.py:14-23)."""

    # tcgen05 flash attention, head_dim 64, reads the packed [B,S,3D] QKV,
    # writes the [B,S,D] context (csrc/attention_kernels.cuh).
    SM100_FLASH = "sm100_flash"
    # Tiled flash attention on the CUDA cores for head_dim 8..256 (the head
    # dims the tensor-core kernels do not build; csrc/attention_simt_kernels.cuh),
    # same packed [B,S,3D] input and [B,S,D] output.
    SM100_SIMT = "sm100_simt"
    # Flash attention for head_dim 8..128 on warp-level tensor-core MMAs
    # (mma.sync m16n8k16; csrc/attention_mma_kernels.cuh), same input and output.
    SM100_MMA = "sm100_mma"


class ProjectionBackend(StrEnum):
    """Per-role projection execution (reference: solution/config.py:26-31)."""

    # tcgen05 GEMM on bf16 shadows of the fp32 master weights.
    SM100_BF16 = "sm100_bf16"


class PrecisionPlan(StrEnum):
    """Projection/cast graphs (reference: solution/config.py:34-44).

    Every projection computes in bf16 with fp32 accumulation; the plans differ in
    the dtype of the two branch updates that feed the fp32 residual stream.
    """

    BF16_CORE = "bf16_core"  # out-proj and FFN-out write bf16 updates
    BF16_CORE_FP32_UPDATES = "bf16_core_fp32_updates"  # they write fp32 updates


class QKVMaterialization(StrEnum):
    """How Q/K/V reach attention (reference: solution/config.py:47-52)."""

    # The attention kernel's TMA reads head tiles straight out of the packed
    # projection output; nothing is split or copied.
    PACKED_BSD = "packed_bsd"


class AttentionOutputBridge(StrEnum):
    """Attention output -> out-projection (reference: solution/config.py:55-60)."""

    ATTENTION_DIRECT_BSD = "attention_direct_bsd"


class FFNBackend(StrEnum):
    """FFN execution (reference: solution/config.py:63-70)."""

    # FFN-in GEMM with a bias + exact-erf GELU epilogue, then the FFN-out GEMM.
    SM100_LINEAR_GELU = "sm100_linear_gelu"
    # The whole MLP fused through its residual + LayerNorm boundary, d_model
    # 32/64/128 (csrc/boundary_kernels.cuh; reference value
    # "triton_fused_mlp_boundary").  Requires the SM100_LINEAR_MIXED boundary.
    SM100_FUSED_MLP_BOUNDARY = "sm100_fused_mlp_boundary"


class ResidualNormBackend(StrEnum):
    """Residual add + LayerNorm (reference: solution/config.py:73-80)."""

    # fp32 residual stream, bf16 normalised output (fp32 at the final boundary).
    SM100_MIXED = "sm100_mixed"
    # The same boundary fused with the projection before it (out-projection and
    # FFN-out), d_model 32/64/128 (csrc/boundary_kernels.cuh; reference value
    # "triton_linear_mixed").
    SM100_LINEAR_MIXED = "sm100_linear_mixed"


class InitialNormBackend(StrEnum):
    """Initial LayerNorm (reference: solution/config.py:83-88)."""

    SM100_BF16 = "sm100_bf16"


class RuntimeBackend(StrEnum):
    """Outer execution schedules (reference: solution/config.py:91-98).

    ``compiled_forward`` is not offered: no torch.compile on the hot path.
    """

    EAGER = "eager"
    CUDA_GRAPH = "cuda_graph"
    BATCH_TILED_CUDA_GRAPH = "batch_tiled_cuda_graph"
    STREAMED = "streamed"
    # The whole forward in one kernel (solution/runtimes/sequence_resident.py):
    # d_model = ffn_dim = 128, 1-4 heads, sequences of 32-128 tokens, no mask.
    SEQUENCE_RESIDENT = "sm100_sequence_resident"


class AttentionOutputLayout(StrEnum):
    """Layouts produced by the selected attention primitive."""

    BHSD = "bhsd"
    BSD = "bsd"


_PROJECTION_FIELDS = (
    "qkv_projection",
    "attention_output_projection",
    "ffn_input_projection",
    "ffn_output_projection",
)

# Roles whose output dtype the precision plan changes (update -> residual).
_FP32_UPDATE_ROLES = {
    PrecisionPlan.BF16_CORE: frozenset(),
    PrecisionPlan.BF16_CORE_FP32_UPDATES: frozenset(
        {"attention_output_projection", "ffn_output_projection"}
    ),
}


def fp32_update_roles(precision_plan: PrecisionPlan) -> frozenset[str]:
    """Projection roles whose output is written in fp32 under this plan."""

    return _FP32_UPDATE_ROLES[PrecisionPlan(precision_plan)]


def _positive_int(value: object, *, field: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ValueError(f"{field} must be a positive integer")
    return value


def _mapping(value: object, *, field: str) -> dict[str, Any]:
    if not isinstance(value, dict):
        raise TypeError(f"{field} must be an object")
    return value


def _exact_fields(value: dict[str, Any], expected: frozenset[str], *, field: str) -> None:
    missing = expected - set(value)
    unknown = set(value) - expected
    if missing or unknown:
        raise ValueError(
            f"invalid {field} fields; missing={sorted(missing)}; unknown={sorted(unknown)}"
        )


# Kernel variants compiled into libb200tx.  Launch parameters outside these
# sets are rejected by the dataclasses, so a search never proposes a variant
# that does not exist.
# (tile_m, tile_n, tile_k, stages) -> libb200tx GEMM variant:
#   (128, 256, 64, 4): one CTA per SM (B200TX_GEMM_1SM)
#   (256, 256, 64, 6): CTA pairs sharing each tile through cta_group::2 (B200TX_GEMM_PAIR)
#   (64, 64, 64, 1):   small problems, 64x64 tiles on warp-level MMAs (B200TX_GEMM_WARP)
SM100_GEMM_VARIANT_CODES = {(128, 256, 64, 4): 0, (256, 256, 64, 6): 1, (64, 64, 64, 1): 2}
SM100_GEMM_VARIANTS = frozenset(SM100_GEMM_VARIANT_CODES)
# (block_m, block_n, kv_stages) -> libb200tx attention variant:
#   (256, 128, 3): two 128-row query tiles per CTA, P kept in TMEM (B200TX_ATTN_PAIRED)
#   (128, 128, 3): one query tile per CTA, P staged through shared memory (B200TX_ATTN_SINGLE)
#   (512, 64, 6):  four query tiles per CTA, 64-row KV tiles, P in TMEM (B200TX_ATTN_QUAD)
#   (256, 64, 8):  persistent grid, two query tiles per work item, double-buffered
#                  scores, 8-slot KV rings (B200TX_ATTN_PERSISTENT)
#   (256, 64, 4):  two query tiles per CTA, 64-row KV tiles, 4-slot KV rings, two CTAs
#                  per SM (B200TX_ATTN_DUO)
#   (256, 128, 4): persistent, two query tiles per work item against 128-row KV
#                  tiles with S, P and O in separate TMEM columns, 4-slot KV rings
#                  (B200TX_ATTN_PINGPONG)
SM100_ATTENTION_VARIANTS = {
    (256, 128, 3): 0,
    (128, 128, 3): 1,
    (512, 64, 6): 2,
    (256, 64, 8): 3,
    (256, 64, 4): 4,
    (256, 128, 4): 5,
}
SM100_NORM_ROWS_PER_CTA = frozenset({8})


@dataclass(frozen=True, slots=True)
class Sm100GemmParams:
    """Tile shape of the tcgen05 GEMM (csrc/gemm_kernels.cuh)."""

    tile_m: int = 256
    tile_n: int = 256
    tile_k: int = 64
    stages: int = 6

    _FIELDS: ClassVar[frozenset[str]] = frozenset({"tile_m", "tile_n", "tile_k", "stages"})

    def __post_init__(self) -> None:
        for name in ("tile_m", "tile_n", "tile_k", "stages"):
            _positive_int(getattr(self, name), field=name)
        key = (self.tile_m, self.tile_n, self.tile_k, self.stages)
        if key not in SM100_GEMM_VARIANTS:
            raise ValueError(f"no sm100 GEMM variant is built for tile {key}")

    @property
    def kernel_variant(self) -> int:
        """The libb200tx GEMM variant code (B200TX_GEMM_1SM / _PAIR / _WARP)."""

        return SM100_GEMM_VARIANT_CODES[(self.tile_m, self.tile_n, self.tile_k, self.stages)]

    def to_dict(self) -> dict[str, int]:
        return {
            "tile_m": self.tile_m,
            "tile_n": self.tile_n,
            "tile_k": self.tile_k,
            "stages": self.stages,
        }

    @classmethod
    def from_dict(cls, payload: object) -> Sm100GemmParams:
        value = _mapping(payload, field="gemm launch")
        _exact_fields(value, cls._FIELDS, field="gemm launch")
        return cls(**value)


@dataclass(frozen=True, slots=True)
class Sm100AttentionParams:
    """Tile shape of the tcgen05 flash attention (csrc/attention_kernels.cuh)."""

    block_m: int = 512
    block_n: int = 64
    kv_stages: int = 6

    _FIELDS: ClassVar[frozenset[str]] = frozenset({"block_m", "block_n", "kv_stages"})

    def __post_init__(self) -> None:
        for name in ("block_m", "block_n", "kv_stages"):
            _positive_int(getattr(self, name), field=name)
        key = (self.block_m, self.block_n, self.kv_stages)
        if key not in SM100_ATTENTION_VARIANTS:
            raise ValueError(f"no sm100 attention variant is built for {key}")

    def to_dict(self) -> dict[str, int]:
        return {"block_m": self.block_m, "block_n": self.block_n, "kv_stages": self.kv_stages}

    @property
    def kernel_variant(self) -> int:
        """The libb200tx attention variant code (B200TX_ATTN_PAIRED / _SINGLE / _QUAD / _PERSISTENT / _DUO)."""

        return SM100_ATTENTION_VARIANTS[(self.block_m, self.block_n, self.kv_stages)]

    @classmethod
    def from_dict(cls, payload: object) -> Sm100AttentionParams:
        value = _mapping(payload, field="attention launch")
        _exact_fields(value, cls._FIELDS, field="attention launch")
        return cls(**value)


@dataclass(frozen=True, slots=True)
class Sm100NormParams:
    """Rows per CTA of the warp-per-row LayerNorm (csrc/norm_kernels.cuh)."""

    rows_per_cta: int = 8

    _FIELDS: ClassVar[frozenset[str]] = frozenset({"rows_per_cta"})

    def __post_init__(self) -> None:
        _positive_int(self.rows_per_cta, field="rows_per_cta")
        if self.rows_per_cta not in SM100_NORM_ROWS_PER_CTA:
            raise ValueError(f"no sm100 norm variant is built for rows_per_cta={self.rows_per_cta}")

    def to_dict(self) -> dict[str, int]:
        return {"rows_per_cta": self.rows_per_cta}

    @classmethod
    def from_dict(cls, payload: object) -> Sm100NormParams:
        value = _mapping(payload, field="norm launch")
        _exact_fields(value, cls._FIELDS, field="norm launch")
        return cls(**value)


@dataclass(frozen=True, slots=True)
class ProgramConfig:
    """High-level execution structure (reference: solution/config.py:389-487)."""

    attention: AttentionBackend
    qkv_projection: ProjectionBackend
    attention_output_projection: ProjectionBackend
    ffn_input_projection: ProjectionBackend
    ffn_output_projection: ProjectionBackend
    precision_plan: PrecisionPlan
    qkv_materialization: QKVMaterialization
    attention_output_bridge: AttentionOutputBridge
    ffn: FFNBackend
    residual_norm: ResidualNormBackend
    initial_norm: InitialNormBackend = InitialNormBackend.SM100_BF16

    _FIELDS: ClassVar[frozenset[str]] = frozenset(
        {
            "attention",
            "qkv_projection",
            "attention_output_projection",
            "ffn_input_projection",
            "ffn_output_projection",
            "precision_plan",
            "qkv_materialization",
            "attention_output_bridge",
            "ffn",
            "residual_norm",
            "initial_norm",
        }
    )

    def __post_init__(self) -> None:
        object.__setattr__(self, "attention", AttentionBackend(self.attention))
        for name in _PROJECTION_FIELDS:
            object.__setattr__(self, name, ProjectionBackend(getattr(self, name)))
        object.__setattr__(self, "precision_plan", PrecisionPlan(self.precision_plan))
        object.__setattr__(
            self, "qkv_materialization", QKVMaterialization(self.qkv_materialization)
        )
        object.__setattr__(
            self, "attention_output_bridge", AttentionOutputBridge(self.attention_output_bridge)
        )
        object.__setattr__(self, "ffn", FFNBackend(self.ffn))
        object.__setattr__(self, "residual_norm", ResidualNormBackend(self.residual_norm))
        object.__setattr__(self, "initial_norm", InitialNormBackend(self.initial_norm))
        # The packed-BSD materialisation is only readable by the sm100 flash
        # kernel, which always writes BSD: keep the pairing explicit so a
        # future variant cannot silently mismatch.
        sm100_attention = (AttentionBackend.SM100_FLASH, AttentionBackend.SM100_SIMT, AttentionBackend.SM100_MMA)
        if (
            self.qkv_materialization is QKVMaterialization.PACKED_BSD
            and self.attention not in sm100_attention
        ):
            raise ValueError("packed_bsd QKV requires an sm100 attention")
        if (
            self.attention_output_bridge is AttentionOutputBridge.ATTENTION_DIRECT_BSD
            and self.attention not in sm100_attention
        ):
            raise ValueError("attention_direct_bsd requires an attention that writes BSD")

    def to_dict(self) -> dict[str, str]:
        return {
            "attention": self.attention.value,
            "qkv_projection": self.qkv_projection.value,
            "attention_output_projection": self.attention_output_projection.value,
            "ffn_input_projection": self.ffn_input_projection.value,
            "ffn_output_projection": self.ffn_output_projection.value,
            "precision_plan": self.precision_plan.value,
            "qkv_materialization": self.qkv_materialization.value,
            "attention_output_bridge": self.attention_output_bridge.value,
            "ffn": self.ffn.value,
            "residual_norm": self.residual_norm.value,
            "initial_norm": self.initial_norm.value,
        }

    @classmethod
    def from_dict(cls, payload: object) -> ProgramConfig:
        value = _mapping(payload, field="program")
        _exact_fields(value, cls._FIELDS, field="program")
        return cls(**value)


def _optional(value: Any, cls: type, field: str) -> Any:
    if value is not None and not isinstance(value, cls):
        raise TypeError(f"{field} must be {cls.__name__} or None")
    return value


@dataclass(frozen=True, slots=True)
class ScheduleConfig:
    """Runtime and launch parameters (reference: solution/config.py:490-669)."""

    runtime: RuntimeBackend
    attention_launch: Sm100AttentionParams | None = None
    qkv_launch: Sm100GemmParams | None = None
    attention_output_projection_launch: Sm100GemmParams | None = None
    residual_norm_launch: Sm100NormParams | None = None
    initial_norm_launch: Sm100NormParams | None = None
    ffn_launch: Sm100GemmParams | None = None  # FFN-out projection
    ffn_input_launch: Sm100GemmParams | None = None  # FFN-in projection + GELU
    batch_tile_size: int | None = None
    microbatch_size: int | None = None
    reuse_unchanged_input: bool = False

    _FIELDS: ClassVar[frozenset[str]] = frozenset(
        {
            "runtime",
            "attention_launch",
            "qkv_launch",
            "attention_output_projection_launch",
            "residual_norm_launch",
            "initial_norm_launch",
            "ffn_launch",
            "ffn_input_launch",
            "batch_tile_size",
            "microbatch_size",
            "reuse_unchanged_input",
        }
    )

    def __post_init__(self) -> None:
        runtime = RuntimeBackend(self.runtime)
        object.__setattr__(self, "runtime", runtime)
        _optional(self.attention_launch, Sm100AttentionParams, "attention_launch")
        for name in (
            "qkv_launch",
            "attention_output_projection_launch",
            "ffn_launch",
            "ffn_input_launch",
        ):
            _optional(getattr(self, name), Sm100GemmParams, name)
        for name in ("residual_norm_launch", "initial_norm_launch"):
            _optional(getattr(self, name), Sm100NormParams, name)
        if runtime is RuntimeBackend.BATCH_TILED_CUDA_GRAPH:
            object.__setattr__(
                self,
                "batch_tile_size",
                _positive_int(self.batch_tile_size, field="batch_tile_size"),
            )
        elif self.batch_tile_size is not None:
            raise ValueError("batch_tile_size is valid only for batch_tiled_cuda_graph")
        if runtime is RuntimeBackend.STREAMED:
            object.__setattr__(
                self,
                "microbatch_size",
                _positive_int(self.microbatch_size, field="microbatch_size"),
            )
        elif self.microbatch_size is not None:
            raise ValueError("microbatch_size is valid only for the streamed runtime")
        if not isinstance(self.reuse_unchanged_input, bool):
            raise TypeError("reuse_unchanged_input must be a bool")
        if self.reuse_unchanged_input and runtime is not RuntimeBackend.CUDA_GRAPH:
            raise ValueError("reuse_unchanged_input is valid only for the cuda_graph runtime")

    def to_dict(self) -> dict[str, Any]:
        def dump(value: Any) -> Any:
            return None if value is None else value.to_dict()

        return {
            "runtime": self.runtime.value,
            "attention_launch": dump(self.attention_launch),
            "qkv_launch": dump(self.qkv_launch),
            "attention_output_projection_launch": dump(self.attention_output_projection_launch),
            "residual_norm_launch": dump(self.residual_norm_launch),
            "initial_norm_launch": dump(self.initial_norm_launch),
            "ffn_launch": dump(self.ffn_launch),
            "ffn_input_launch": dump(self.ffn_input_launch),
            "batch_tile_size": self.batch_tile_size,
            "microbatch_size": self.microbatch_size,
            "reuse_unchanged_input": self.reuse_unchanged_input,
        }

    @classmethod
    def from_dict(cls, payload: object) -> ScheduleConfig:
        value = _mapping(payload, field="schedule")
        _exact_fields(value, cls._FIELDS, field="schedule")

        def load(key: str, parser: Any) -> Any:
            return None if value[key] is None else parser(value[key])

        return cls(
            runtime=value["runtime"],
            attention_launch=load("attention_launch", Sm100AttentionParams.from_dict),
            qkv_launch=load("qkv_launch", Sm100GemmParams.from_dict),
            attention_output_projection_launch=load(
                "attention_output_projection_launch", Sm100GemmParams.from_dict
            ),
            residual_norm_launch=load("residual_norm_launch", Sm100NormParams.from_dict),
            initial_norm_launch=load("initial_norm_launch", Sm100NormParams.from_dict),
            ffn_launch=load("ffn_launch", Sm100GemmParams.from_dict),
            ffn_input_launch=load("ffn_input_launch", Sm100GemmParams.from_dict),
            batch_tile_size=value["batch_tile_size"],
            microbatch_size=value["microbatch_size"],
            reuse_unchanged_input=value["reuse_unchanged_input"],
        )


@functools.lru_cache(maxsize=256)
def _sha256_of(text: str) -> str:
    return hashlib.sha256(text.encode("utf-8")).hexdigest()


@dataclass(frozen=True, slots=True)
class ConfigSpec:
    """Canonical program plus schedule (reference: solution/config.py:672-785)."""

    program: ProgramConfig
    schedule: ScheduleConfig
    schema_version: int = CONFIG_SCHEMA_VERSION
    # The canonical JSON, computed once: the config is immutable, and the
    # forward reads config_id on every call.
    _canonical: str = field(default="", init=False, repr=False, compare=False)

    _FIELDS: ClassVar[frozenset[str]] = frozenset({"schema_version", "program", "schedule"})

    def __post_init__(self) -> None:
        if self.schema_version != CONFIG_SCHEMA_VERSION:
            raise ValueError(f"schema_version must be {CONFIG_SCHEMA_VERSION}")
        if not isinstance(self.program, ProgramConfig):
            raise TypeError("program must be ProgramConfig")
        if not isinstance(self.schedule, ScheduleConfig):
            raise TypeError("schedule must be ScheduleConfig")
        # Every sm100 primitive is a parameterised kernel: its launch record
        # must be present (reference rule: launch present exactly for a
        # parameterised backend, solution/config.py:713-758).
        # A fused boundary runs the row-parallel projections itself: their
        # GEMM launch records are absent (reference: solution/config.py:706-717).
        fused = self.program.residual_norm is ResidualNormBackend.SM100_LINEAR_MIXED
        required = {
            "attention_launch": self.program.attention is AttentionBackend.SM100_FLASH,
            "qkv_launch": self.program.qkv_projection is ProjectionBackend.SM100_BF16,
            "attention_output_projection_launch": (
                self.program.attention_output_projection is ProjectionBackend.SM100_BF16 and not fused
            ),
            "ffn_input_launch": self.program.ffn is FFNBackend.SM100_LINEAR_GELU,
            "ffn_launch": self.program.ffn_output_projection is ProjectionBackend.SM100_BF16 and not fused,
            "residual_norm_launch": self.program.residual_norm
            in (ResidualNormBackend.SM100_MIXED, ResidualNormBackend.SM100_LINEAR_MIXED),
            "initial_norm_launch": self.program.initial_norm is InitialNormBackend.SM100_BF16,
        }
        for name, needed in required.items():
            if needed != (getattr(self.schedule, name) is not None):
                raise ValueError(f"{name} must be present exactly for its sm100 primitive")

    @property
    def attention_output_layout(self) -> AttentionOutputLayout:
        if self.program.attention_output_bridge is AttentionOutputBridge.ATTENTION_DIRECT_BSD:
            return AttentionOutputLayout.BSD
        return AttentionOutputLayout.BHSD

    def to_dict(self) -> dict[str, Any]:
        return {
            "schema_version": self.schema_version,
            "program": self.program.to_dict(),
            "schedule": self.schedule.to_dict(),
        }

    def canonical_json(self) -> str:
        if not self._canonical:
            object.__setattr__(
                self,
                "_canonical",
                json.dumps(self.to_dict(), ensure_ascii=True, allow_nan=False, sort_keys=True, separators=(",", ":")),
            )
        return self._canonical

    @property
    def sha256(self) -> str:
        return _sha256_of(self.canonical_json())

    @property
    def config_id(self) -> str:
        return f"cfg-{self.sha256}"

    @classmethod
    def from_dict(cls, payload: object) -> ConfigSpec:
        value = _mapping(payload, field="config")
        _exact_fields(value, cls._FIELDS, field="config")
        return cls(
            schema_version=value["schema_version"],
            program=ProgramConfig.from_dict(value["program"]),
            schedule=ScheduleConfig.from_dict(value["schedule"]),
        )


# Boundary fusion choices of default_program / default_schedule: None (the
# unfused program), "linear" (SM100_LINEAR_MIXED: out-projection and FFN-out
# fused with their residual LayerNorm) or "mlp" (SM100_LINEAR_MIXED plus the
# whole MLP fused, SM100_FUSED_MLP_BOUNDARY).
BOUNDARY_FUSIONS = (None, "linear", "mlp")


def _check_fusion(fused_boundary: str | None) -> None:
    if fused_boundary not in BOUNDARY_FUSIONS:
        raise ValueError(f"fused_boundary must be one of {BOUNDARY_FUSIONS}")


def default_program(
    precision_plan: PrecisionPlan = PrecisionPlan.BF16_CORE,
    attention: AttentionBackend = AttentionBackend.SM100_FLASH,
    *,
    fused_boundary: str | None = None,
) -> ProgramConfig:
    """The sm100 program: every primitive is a libb200tx kernel."""

    _check_fusion(fused_boundary)
    return ProgramConfig(
        attention=attention,
        qkv_projection=ProjectionBackend.SM100_BF16,
        attention_output_projection=ProjectionBackend.SM100_BF16,
        ffn_input_projection=ProjectionBackend.SM100_BF16,
        ffn_output_projection=ProjectionBackend.SM100_BF16,
        precision_plan=precision_plan,
        qkv_materialization=QKVMaterialization.PACKED_BSD,
        attention_output_bridge=AttentionOutputBridge.ATTENTION_DIRECT_BSD,
        ffn=FFNBackend.SM100_FUSED_MLP_BOUNDARY if fused_boundary == "mlp" else FFNBackend.SM100_LINEAR_GELU,
        residual_norm=(
            ResidualNormBackend.SM100_MIXED if fused_boundary is None else ResidualNormBackend.SM100_LINEAR_MIXED
        ),
        initial_norm=InitialNormBackend.SM100_BF16,
    )


def default_schedule(
    runtime: RuntimeBackend = RuntimeBackend.EAGER,
    *,
    batch_tile_size: int | None = None,
    microbatch_size: int | None = None,
    reuse_unchanged_input: bool = False,
    attention: AttentionBackend = AttentionBackend.SM100_FLASH,
    fused_boundary: str | None = None,
) -> ScheduleConfig:
    _check_fusion(fused_boundary)
    gemm = Sm100GemmParams()
    return ScheduleConfig(
        runtime=runtime,
        attention_launch=Sm100AttentionParams() if attention is AttentionBackend.SM100_FLASH else None,
        qkv_launch=gemm,
        attention_output_projection_launch=None if fused_boundary else gemm,
        residual_norm_launch=Sm100NormParams(),
        initial_norm_launch=Sm100NormParams(),
        ffn_launch=None if fused_boundary else gemm,
        ffn_input_launch=None if fused_boundary == "mlp" else gemm,
        batch_tile_size=batch_tile_size,
        microbatch_size=microbatch_size,
        reuse_unchanged_input=reuse_unchanged_input,
    )


def default_attention(head_dim: int | None) -> AttentionBackend:
    """The tcgen05 kernels for head_dim 64 (or unknown), the warp-MMA kernel for
    8, 16, 32 and 128, else the CUDA-core one (256)."""

    if head_dim in (None, 64):
        return AttentionBackend.SM100_FLASH
    if head_dim in (8, 16, 32, 128):
        return AttentionBackend.SM100_MMA
    return AttentionBackend.SM100_SIMT


def portable_config(*, head_dim: int | None = None) -> ConfigSpec:
    """The default program under the eager schedule.

    In the reference this is the torch fallback (solution/config.py:788-806);
    here there is no fallback, so "portable" means the sm100 program with no
    shape-specific schedule (its attention chosen by head_dim).
    """

    attention = default_attention(head_dim)
    return ConfigSpec(
        program=default_program(attention=attention), schedule=default_schedule(attention=attention)
    )


def portable_streamed_config(*, microbatch_size: int = 1) -> ConfigSpec:
    """The default program under the streamed schedule (reference :809-818)."""

    return ConfigSpec(
        program=default_program(),
        schedule=default_schedule(RuntimeBackend.STREAMED, microbatch_size=microbatch_size),
    )


__all__ = [
    "CONFIG_SCHEMA_VERSION",
    "SM100_ATTENTION_VARIANTS",
    "SM100_GEMM_VARIANTS",
    "SM100_NORM_ROWS_PER_CTA",
    "AttentionBackend",
    "AttentionOutputBridge",
    "AttentionOutputLayout",
    "ConfigSpec",
    "BOUNDARY_FUSIONS",
    "FFNBackend",
    "InitialNormBackend",
    "PrecisionPlan",
    "ProgramConfig",
    "ProjectionBackend",
    "QKVMaterialization",
    "ResidualNormBackend",
    "RuntimeBackend",
    "ScheduleConfig",
    "Sm100AttentionParams",
    "Sm100GemmParams",
    "Sm100NormParams",
    "default_attention",
    "default_program",
    "default_schedule",
    "fp32_update_roles",
    "portable_config",
    "portable_streamed_config",
]
