"""Search space over the built sm100 kernel variants, for the program search.

The reference's autotune loop (autotune/optimization_loop.py) samples
``ConfigSpec`` candidates from ``ProgramSearchSpace`` (autotune/search_space.py:
1589-1693) and keeps those its ``PlanBuilder`` accepts.  This module provides
the same surface -- ``SearchContext``, ``ParameterDomain``, ``StructureSpec``,
``BranchSpace`` and ``ProgramSearchSpace`` with the same method names -- but
its choices are the sm100 programs and the kernel variants compiled into
libb200tx, so every candidate it yields is runnable on a B200:

* structure (one branch each): attention backend (tensor-core flash kernels
  or the CUDA-core kernel for other head dims) x precision plan x runtime
  (resident scope: eager, CUDA graph, batch-tiled CUDA graph; streamed scope:
  the streamed runtime, reference autotune/shape14_search_space.py:26-156);
* parameters of a branch: the attention variant (``Sm100AttentionParams``
  tile), one GEMM variant per projection role (``Sm100GemmParams`` tile), and
  the runtime's own knob (batch tile, microbatch, input reuse).

A branch's cardinality is the product of its domain sizes; ``config_at`` /
``index_for`` map between configs and a mixed-radix index, so an exhaustive
sweep (``autotune.sweep``) and a sampler (``suggest`` with an Optuna-like
trial) see the same space.  The Optuna loop itself is not part of this
package.
"""

from __future__ import annotations

import hashlib
import json
import random
from collections.abc import Iterable, Iterator, Mapping, Sequence
from dataclasses import dataclass, field, replace
from typing import Any, Protocol, Union

from solution.config import (
    BOUNDARY_FUSIONS,
    SM100_ATTENTION_VARIANTS,
    AttentionBackend,
    SM100_GEMM_VARIANTS,
    ConfigSpec,
    FFNBackend,
    PrecisionPlan,
    ResidualNormBackend,
    RuntimeBackend,
    Sm100AttentionParams,
    Sm100GemmParams,
    default_attention,
    default_program,
    default_schedule,
    portable_config,
)

Scalar = Union[str, int, bool]
DEFAULT_MAX_STRUCTURE_BRANCHES = 16

_GEMM_ROLES = (
    ("qkv_tile", "qkv_launch"),
    ("attention_output_projection_tile", "attention_output_projection_launch"),
    ("ffn_input_tile", "ffn_input_launch"),
    ("ffn_output_tile", "ffn_launch"),
)
_RESIDENT_RUNTIMES = (
    RuntimeBackend.EAGER,
    RuntimeBackend.CUDA_GRAPH,
    RuntimeBackend.BATCH_TILED_CUDA_GRAPH,
)


class TrialLike(Protocol):
    """Narrow Optuna Trial surface (reference autotune/search_space.py:156-163)."""

    def suggest_categorical(self, name: str, choices: Sequence[Scalar]) -> Scalar: ...


class CompilationResultLike(Protocol):
    @property
    def accepted(self) -> bool: ...


class PlanBuilderLike(Protocol):
    def evaluate(self, config: ConfigSpec, context: Any, hardware: Any | None = None) -> CompilationResultLike: ...


@dataclass(frozen=True, slots=True)
class SearchContext:
    """Compiler inputs plus the logical batch (reference :181-208)."""

    execution_context: Any
    scope: str
    hardware: Any | None = None
    logical_batch_size: int | None = None

    def __post_init__(self) -> None:
        if self.scope not in {"resident", "streamed"}:
            raise ValueError("scope must be resident or streamed")
        if self.logical_batch_size is not None and (
            isinstance(self.logical_batch_size, bool)
            or not isinstance(self.logical_batch_size, int)
            or self.logical_batch_size <= 0
        ):
            raise ValueError("logical_batch_size must be a positive integer")

    @property
    def batch_size(self) -> int:
        if self.logical_batch_size is not None:
            return self.logical_batch_size
        value = getattr(self.execution_context, "batch_size", None)
        if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
            raise ValueError("compilation context has no valid batch_size")
        return value


@dataclass(frozen=True, slots=True)
class ParameterDomain:
    """One finite parameter domain (reference :211-229)."""

    name: str
    choices: tuple[Scalar, ...]
    default: Scalar

    def __post_init__(self) -> None:
        if not self.name:
            raise ValueError("parameter name must not be empty")
        if not self.choices:
            raise ValueError(f"parameter {self.name!r} needs at least one choice")
        if len(set(self.choices)) != len(self.choices):
            raise ValueError(f"parameter {self.name!r} has duplicate choices")
        if self.default not in self.choices:
            raise ValueError(f"default for {self.name!r} is outside its domain")

    def suggest(self, trial: TrialLike) -> Scalar:
        return trial.suggest_categorical(self.name, self.choices)


def _digest(value: object) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True).encode()).hexdigest()[:16]


def _tile_name(key: tuple[int, ...]) -> str:
    return "x".join(str(v) for v in key)


def _tile_key(value: Scalar) -> tuple[int, ...]:
    return tuple(int(v) for v in str(value).split("x"))


_ATTENTION_CHOICES = tuple(_tile_name(k) for k in SM100_ATTENTION_VARIANTS)
_GEMM_CHOICES = tuple(_tile_name(k) for k in sorted(SM100_GEMM_VARIANTS, reverse=True))
_DEFAULT_ATTENTION = _tile_name(
    (Sm100AttentionParams().block_m, Sm100AttentionParams().block_n, Sm100AttentionParams().kv_stages)
)
_DEFAULT_GEMM = _tile_name(
    (Sm100GemmParams().tile_m, Sm100GemmParams().tile_n, Sm100GemmParams().tile_k, Sm100GemmParams().stages)
)


@dataclass(frozen=True, slots=True)
class StructureSpec:
    """The branch-defining program facts (reference :244-327)."""

    precision_plan: PrecisionPlan
    runtime: RuntimeBackend
    attention: AttentionBackend = AttentionBackend.SM100_FLASH
    # Block-boundary fusion (None, "linear", "mlp"; see default_program).
    boundary: str | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "precision_plan", PrecisionPlan(self.precision_plan))
        object.__setattr__(self, "runtime", RuntimeBackend(self.runtime))
        object.__setattr__(self, "attention", AttentionBackend(self.attention))
        if self.boundary not in BOUNDARY_FUSIONS:
            raise ValueError(f"boundary must be one of {BOUNDARY_FUSIONS}")

    def to_dict(self) -> dict[str, str]:
        value = {
            "attention": self.attention.value,
            "precision_plan": self.precision_plan.value,
            "runtime": self.runtime.value,
        }
        if self.boundary is not None:  # unfused structures keep their earlier identity
            value["boundary"] = self.boundary
        return value

    @property
    def branch_id(self) -> str:
        return _digest(self.to_dict())

    @property
    def portable(self) -> bool:
        """The eager bf16-core tensor-core branch: the default program's own structure."""

        return (
            self.precision_plan is PrecisionPlan.BF16_CORE
            and self.runtime is RuntimeBackend.EAGER
            and self.attention is AttentionBackend.SM100_FLASH
            and self.boundary is None
        )

    @classmethod
    def from_config(cls, config: ConfigSpec) -> StructureSpec:
        program = config.program
        boundary = None
        if program.residual_norm is ResidualNormBackend.SM100_LINEAR_MIXED:
            boundary = "mlp" if program.ffn is FFNBackend.SM100_FUSED_MLP_BOUNDARY else "linear"
        return cls(program.precision_plan, config.schedule.runtime, program.attention, boundary)


def _fused_launches(boundary: str | None) -> frozenset[str]:
    """Schedule launch fields a fused boundary makes absent."""

    if boundary is None:
        return frozenset()
    fused = {"attention_output_projection_launch", "ffn_launch"}
    if boundary == "mlp":
        fused.add("ffn_input_launch")
    return frozenset(fused)


def _divisors(n: int, *, below: int | None = None) -> tuple[int, ...]:
    limit = n if below is None else below
    return tuple(d for d in range(1, n + 1) if n % d == 0 and d <= limit)


def _domains_for_structure(structure: StructureSpec, context: SearchContext) -> tuple[ParameterDomain, ...]:
    if structure.runtime is RuntimeBackend.SEQUENCE_RESIDENT:
        return ()  # one kernel for the whole forward: no per-primitive launch to tune
    domains = []
    if structure.attention is AttentionBackend.SM100_FLASH:
        domains.append(ParameterDomain("attention_tile", _ATTENTION_CHOICES, _DEFAULT_ATTENTION))
    domains += [
        ParameterDomain(name, _GEMM_CHOICES, _DEFAULT_GEMM)
        for name, launch_field in _GEMM_ROLES
        if launch_field not in _fused_launches(structure.boundary)
    ]
    batch = context.batch_size
    if structure.runtime is RuntimeBackend.BATCH_TILED_CUDA_GRAPH:
        tiles = tuple(d for d in _divisors(batch) if d < batch)
        if tiles:
            domains.append(ParameterDomain("batch_tile_size", tiles, tiles[-1]))
    elif structure.runtime is RuntimeBackend.STREAMED:
        micro = _divisors(batch)
        domains.append(ParameterDomain("microbatch_size", micro, micro[len(micro) // 2]))
    elif structure.runtime is RuntimeBackend.CUDA_GRAPH:
        domains.append(ParameterDomain("reuse_unchanged_input", (False, True), False))
    return tuple(domains)


def _structure_specs(context: SearchContext) -> tuple[StructureSpec, ...]:
    runtimes = (RuntimeBackend.STREAMED,) if context.scope == "streamed" else _RESIDENT_RUNTIMES
    specs = []
    for boundary in BOUNDARY_FUSIONS:
        for attention in AttentionBackend:
            for plan in PrecisionPlan:
                for runtime in runtimes:
                    if runtime is RuntimeBackend.BATCH_TILED_CUDA_GRAPH and context.batch_size < 2:
                        continue
                    specs.append(StructureSpec(plan, runtime, attention, boundary))
    ctx = context.execution_context
    if context.scope == "resident" and _sequence_resident_eligible(ctx):
        # The whole forward in one kernel: one structure, the program's
        # primitives being the kernel's own.
        head_dim = ctx.d_model // ctx.num_heads
        specs.append(StructureSpec(PrecisionPlan.BF16_CORE, RuntimeBackend.SEQUENCE_RESIDENT,
                                   default_attention(head_dim), None))
    return tuple(specs)


def _sequence_resident_eligible(ctx: Any) -> bool:
    from solution.runtimes.sequence_resident import sequence_resident_supported

    try:
        return sequence_resident_supported(
            d_model=ctx.d_model, ffn_dim=ctx.ffn_dim, num_heads=ctx.num_heads, seq_len=ctx.seq_len,
            num_layers=ctx.num_layers, causal=bool(ctx.causal),
        ) is None and not ctx.has_valid_token_mask
    except (AttributeError, TypeError, ZeroDivisionError):
        return False


@dataclass(frozen=True, slots=True)
class BranchSpace:
    """One structure and its parameter domains (reference :448-763)."""

    structure: StructureSpec
    domains: tuple[ParameterDomain, ...]
    scope: str
    witness_parameters: tuple[tuple[str, Scalar], ...] = field(default=())

    def __post_init__(self) -> None:
        names = [d.name for d in self.domains]
        if len(set(names)) != len(names):
            raise ValueError("duplicate parameter names in a branch")

    @property
    def branch_id(self) -> str:
        return self.structure.branch_id

    @property
    def cardinality(self) -> int:
        total = 1
        for domain in self.domains:
            total *= len(domain.choices)
        return total

    @property
    def parameter_names(self) -> tuple[str, ...]:
        return tuple(d.name for d in self.domains)

    def parameters_at(self, index: int) -> dict[str, Scalar]:
        if isinstance(index, bool) or not isinstance(index, int) or not 0 <= index < self.cardinality:
            raise IndexError(f"index {index} outside [0, {self.cardinality})")
        values: dict[str, Scalar] = {}
        for domain in reversed(self.domains):
            index, digit = divmod(index, len(domain.choices))
            values[domain.name] = domain.choices[digit]
        return {name: values[name] for name in self.parameter_names}

    def config_at(self, index: int) -> ConfigSpec:
        return self.build(self.parameters_at(index))

    def index_for(self, config: ConfigSpec) -> int | None:
        parameters = self.parameters_for(config)
        if parameters is None:
            return None
        index = 0
        for domain in self.domains:
            index = index * len(domain.choices) + domain.choices.index(parameters[domain.name])
        return index

    def default_parameters(self) -> dict[str, Scalar]:
        if self.witness_parameters:
            return dict(self.witness_parameters)
        return {d.name: d.default for d in self.domains}

    def default_config(self) -> ConfigSpec:
        return self.build(self.default_parameters())

    def suggest_parameters(self, trial: TrialLike) -> dict[str, Scalar]:
        return {d.name: d.suggest(trial) for d in self.domains}

    def suggest(self, trial: TrialLike) -> ConfigSpec:
        return self.build(self.suggest_parameters(trial))

    def configs(self) -> Iterator[ConfigSpec]:
        for index in range(self.cardinality):
            yield self.config_at(index)

    def build(self, parameters: Mapping[str, Scalar]) -> ConfigSpec:
        missing = set(self.parameter_names) - set(parameters)
        unknown = set(parameters) - set(self.parameter_names)
        if missing or unknown:
            raise ValueError(f"parameters: missing={sorted(missing)} unknown={sorted(unknown)}")
        for domain in self.domains:
            if parameters[domain.name] not in domain.choices:
                raise ValueError(f"{domain.name}={parameters[domain.name]!r} is outside its domain")
        runtime = self.structure.runtime
        schedule = default_schedule(
            runtime,
            batch_tile_size=parameters.get("batch_tile_size") if runtime is RuntimeBackend.BATCH_TILED_CUDA_GRAPH else None,
            microbatch_size=parameters.get("microbatch_size") if runtime is RuntimeBackend.STREAMED else None,
            reuse_unchanged_input=bool(parameters.get("reuse_unchanged_input", False)),
            attention=self.structure.attention,
            fused_boundary=self.structure.boundary,
        )
        updates: dict[str, Any] = {}
        if "attention_tile" in parameters:
            m, n, stages = _tile_key(parameters["attention_tile"])
            updates["attention_launch"] = Sm100AttentionParams(block_m=m, block_n=n, kv_stages=stages)
        for name, launch_field in _GEMM_ROLES:
            if name not in parameters:  # a projection the fused boundary runs itself
                continue
            tm, tn, tk, st = _tile_key(parameters[name])
            updates[launch_field] = Sm100GemmParams(tile_m=tm, tile_n=tn, tile_k=tk, stages=st)
        return ConfigSpec(
            program=default_program(
                self.structure.precision_plan, self.structure.attention, fused_boundary=self.structure.boundary
            ),
            schedule=replace(schedule, **updates),
        )

    def parameters_for(self, config: ConfigSpec) -> dict[str, Scalar] | None:
        if StructureSpec.from_config(config) != self.structure:
            return None
        schedule = config.schedule
        values: dict[str, Scalar] = {}
        if "attention_tile" in self.parameter_names:
            a = schedule.attention_launch
            if a is None:
                return None
            values["attention_tile"] = _tile_name((a.block_m, a.block_n, a.kv_stages))
        for name, launch_field in _GEMM_ROLES:
            if name not in self.parameter_names:
                continue
            g = getattr(schedule, launch_field)
            if g is None:
                return None
            values[name] = _tile_name((g.tile_m, g.tile_n, g.tile_k, g.stages))
        if "batch_tile_size" in self.parameter_names:
            values["batch_tile_size"] = schedule.batch_tile_size
        if "microbatch_size" in self.parameter_names:
            values["microbatch_size"] = schedule.microbatch_size
        if "reuse_unchanged_input" in self.parameter_names:
            values["reuse_unchanged_input"] = bool(schedule.reuse_unchanged_input)
        for domain in self.domains:
            if values.get(domain.name) not in domain.choices:
                return None
        try:
            rebuilt = self.build(values)
        except ValueError:
            return None
        return values if rebuilt == config else None


def _with_first_feasible_witness(branch: BranchSpace, accepted: Any) -> BranchSpace | None:
    """The branch with its first accepted parameter set as witness, or None."""

    default = branch.default_parameters()
    if accepted(branch.build(default)):
        return replace(branch, witness_parameters=tuple(default.items()))
    for index in range(branch.cardinality):
        parameters = branch.parameters_at(index)
        if accepted(branch.build(parameters)):
            return replace(branch, witness_parameters=tuple(parameters.items()))
    return None


class ProgramSearchSpace:
    """Legal sm100 branches, filtered by the plan builder (reference :1589-1693)."""

    def __init__(
        self,
        *,
        plan_builder: PlanBuilderLike,
        context: SearchContext,
        max_branches: int = DEFAULT_MAX_STRUCTURE_BRANCHES,
        required_configs: Iterable[ConfigSpec] = (),
        seed: int = 0,
    ) -> None:
        if isinstance(max_branches, bool) or not isinstance(max_branches, int) or max_branches <= 0:
            raise ValueError("max_branches must be a positive integer")
        if isinstance(seed, bool) or not isinstance(seed, int):
            raise TypeError("seed must be an integer")
        self.plan_builder = plan_builder
        self.context = context
        candidates: list[BranchSpace] = []
        for structure in _structure_specs(context):
            branch = BranchSpace(structure, _domains_for_structure(structure, context), context.scope)
            witnessed = _with_first_feasible_witness(branch, self.accepted)
            if witnessed is not None:
                candidates.append(witnessed)
        required_ids = [b.branch_id for b in candidates if b.structure.portable]
        # The default program for this head dim (its attention chosen by
        # head_dim) is always searched, as the portable branch is.
        head_dim = getattr(context.execution_context, "head_dim", None)
        for config in (portable_config(head_dim=head_dim), *required_configs):
            match = next((b for b in candidates if b.parameters_for(config) is not None), None)
            if match is not None and self.accepted(config):
                required_ids.append(match.branch_id)
        if not candidates:
            raise ValueError("plan builder accepted no search branches")
        mandatory = [b for b in candidates if b.branch_id in set(required_ids)]
        optional = [b for b in candidates if b.branch_id not in set(required_ids)]
        random.Random(seed).shuffle(optional)
        chosen = (mandatory + optional)[: max(max_branches, len(mandatory))]
        order = {b.branch_id: i for i, b in enumerate(candidates)}
        self.branches = tuple(sorted(chosen, key=lambda b: order[b.branch_id]))
        self.mandatory_branch_ids = tuple(dict.fromkeys(required_ids))
        self._by_id = {b.branch_id: b for b in self.branches}

    def accepted(self, config: ConfigSpec) -> bool:
        result = self.plan_builder.evaluate(config, self.context.execution_context, self.context.hardware)
        return bool(result.accepted)

    def branch(self, branch_id: str) -> BranchSpace:
        try:
            return self._by_id[branch_id]
        except KeyError as exc:
            raise KeyError(f"unknown branch_id: {branch_id}") from exc

    def branch_for(self, config: ConfigSpec) -> BranchSpace | None:
        for branch in self.branches:
            if branch.parameters_for(config) is not None:
                return branch
        return None

    @property
    def cardinality(self) -> int:
        return sum(b.cardinality for b in self.branches)

    def configs(self, *, accepted_only: bool = True) -> Iterator[ConfigSpec]:
        """Every config of every branch (the plan builder's rejects skipped)."""

        for branch in self.branches:
            for config in branch.configs():
                if not accepted_only or self.accepted(config):
                    yield config


__all__ = [
    "DEFAULT_MAX_STRUCTURE_BRANCHES",
    "BranchSpace",
    "ParameterDomain",
    "PlanBuilderLike",
    "ProgramSearchSpace",
    "SearchContext",
    "StructureSpec",
]
