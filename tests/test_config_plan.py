"""ConfigSpec / PlanBuilder contract on the CPU (no GPU needed).

Mirrors the reference's program tests (tests/solution/test_program_primitives.py
plan/trace equality on a tiny model, rejection codes) for the sm100 program.
"""

from __future__ import annotations

import json
from dataclasses import replace

import pytest
import torch

from solution.config import (
    CONFIG_SCHEMA_VERSION,
    ConfigSpec,
    PrecisionPlan,
    RuntimeBackend,
    ScheduleConfig,
    Sm100AttentionParams,
    Sm100GemmParams,
    Sm100NormParams,
    default_program,
    default_schedule,
    portable_config,
    portable_streamed_config,
)
from solution.plan import ExecutionContext
from solution.plan_builder import (
    CompileRejection,
    ConfigRejectedError,
    ConstraintViolation,
    HardwareCapabilities,
    PlanBuilder,
)


def _context(**overrides: object) -> ExecutionContext:
    base = dict(
        batch_size=2,
        seq_len=128,
        d_model=256,
        num_heads=4,
        causal=True,
        device=torch.device("cuda", 0),
        dtype=torch.float32,
        training=False,
        grad_enabled=False,
        input_contiguous=True,
        has_valid_token_mask=False,
        mask_compatible=True,
        ffn_dim=1024,
        num_layers=2,
    )
    base.update(overrides)
    return ExecutionContext(**base)  # type: ignore[arg-type]


B200 = HardwareCapabilities.sm100()


def _codes(result) -> set[str]:  # noqa: ANN001
    return {v.code for v in result.violations}


def test_round_trip_and_canonical_json() -> None:
    cfg = portable_config()
    payload = json.loads(cfg.canonical_json())
    assert payload["schema_version"] == CONFIG_SCHEMA_VERSION == 5
    again = ConfigSpec.from_dict(payload)
    assert again == cfg
    assert again.config_id == cfg.config_id
    assert cfg.config_id.startswith("cfg-") and len(cfg.config_id) == 4 + 64


def test_config_id_changes_with_schedule() -> None:
    a = portable_config()
    b = ConfigSpec(program=default_program(), schedule=default_schedule(RuntimeBackend.CUDA_GRAPH))
    assert a.config_id != b.config_id


def test_schema_v4_and_unknown_fields_are_rejected() -> None:
    payload = portable_config().to_dict()
    payload["schema_version"] = 4
    with pytest.raises(ValueError):
        ConfigSpec.from_dict(payload)
    payload = portable_config().to_dict()
    payload["program"]["extra"] = "x"
    with pytest.raises(ValueError):
        ConfigSpec.from_dict(payload)
    payload = portable_config().to_dict()
    payload["program"]["attention"] = "triton_streaming_dh64"
    with pytest.raises(ValueError):
        ConfigSpec.from_dict(payload)


def test_launch_params_must_name_a_built_variant() -> None:
    with pytest.raises(ValueError):
        Sm100GemmParams(tile_m=128, tile_n=128, tile_k=64, stages=4)
    with pytest.raises(ValueError):
        Sm100AttentionParams(block_m=64)
    with pytest.raises(ValueError):
        Sm100AttentionParams(block_m=512, block_n=128, kv_stages=6)
    assert Sm100AttentionParams().kernel_variant == 2
    assert Sm100AttentionParams(block_m=256, block_n=128, kv_stages=3).kernel_variant == 0
    assert Sm100AttentionParams(block_m=128, block_n=128, kv_stages=3).kernel_variant == 1
    assert Sm100AttentionParams(block_m=512, block_n=64, kv_stages=6).kernel_variant == 2
    with pytest.raises(ValueError):
        Sm100NormParams(rows_per_cta=4)
    with pytest.raises(ValueError):
        Sm100GemmParams(tile_m=0)


def test_launch_records_required_exactly() -> None:
    schedule = replace(default_schedule(), attention_launch=None)
    with pytest.raises(ValueError, match="attention_launch"):
        ConfigSpec(program=default_program(), schedule=schedule)


def test_schedule_field_rules() -> None:
    with pytest.raises(ValueError):
        ScheduleConfig(runtime=RuntimeBackend.EAGER, batch_tile_size=4)
    with pytest.raises(ValueError):
        ScheduleConfig(runtime=RuntimeBackend.STREAMED)
    with pytest.raises(ValueError):
        ScheduleConfig(runtime=RuntimeBackend.EAGER, reuse_unchanged_input=True)
    with pytest.raises(ValueError):
        ScheduleConfig(runtime="compiled_forward")
    s = ScheduleConfig(runtime=RuntimeBackend.BATCH_TILED_CUDA_GRAPH, batch_tile_size=8)
    assert s.batch_tile_size == 8


def test_plan_accepted_on_sm100_snapshot() -> None:
    result = PlanBuilder().evaluate(portable_config(), _context(), B200)
    assert result.accepted, result.violations
    plan = result.require_plan()
    trace = plan.expected_trace.to_dict()
    assert trace["attention_calls"] == 2
    assert trace["residual_norm_calls"] == 4
    assert trace["initial_norm_calls"] == 1
    assert trace["attention_backend"] == "sm100_flash"
    assert trace["complete"] is True
    described = plan.describe()
    assert described["causal_mask"] == "online_causal"
    assert described["attention_output_layout"] == "bsd"
    assert plan.output_dtype == "float32"


def test_precision_plan_sets_update_dtypes() -> None:
    cfg = ConfigSpec(
        program=default_program(PrecisionPlan.BF16_CORE_FP32_UPDATES), schedule=default_schedule()
    )
    plan = PlanBuilder().build(cfg, _context(), B200)
    assert plan.attention_output_update_dtype == "float32"
    assert plan.ffn_output_update_dtype == "float32"
    plan = PlanBuilder().build(portable_config(), _context(), B200)
    assert plan.attention_output_update_dtype == "bfloat16"


@pytest.mark.parametrize(
    ("overrides", "hardware", "code"),
    [
        ({"device": torch.device("cpu")}, HardwareCapabilities("cpu", None, None, None, True), "requires_cuda"),
        ({}, HardwareCapabilities("cuda", (9, 0), 232448, 132, True), "requires_sm100"),
        ({}, replace(B200, kernel_library=False), "backend_unavailable"),
        ({"training": True}, B200, "requires_inference"),
        ({"grad_enabled": True}, B200, "requires_inference"),
        ({"dtype": torch.float16}, B200, "unsupported_dtype"),
        ({"input_contiguous": False}, B200, "requires_contiguous_input"),
        ({"d_model": 256, "num_heads": 2}, B200, "unsupported_shape"),  # head_dim 128
        ({"d_model": 250, "num_heads": 5}, B200, "unsupported_shape"),
        ({"ffn_dim": 1020}, B200, "unsupported_shape"),
        ({"num_heads": 3}, B200, "not_divisible"),
        ({"seq_len": 0}, B200, "non_positive"),
    ],
)
def test_structured_rejections(overrides: dict, hardware: HardwareCapabilities, code: str) -> None:
    result = PlanBuilder().evaluate(portable_config(), _context(**overrides), hardware)
    assert not result.accepted
    assert code in _codes(result)
    with pytest.raises(ConfigRejectedError):
        result.require_plan()


def test_padding_masks_need_a_mask_reading_attention_variant() -> None:
    masked = _context(has_valid_token_mask=True)
    plan = PlanBuilder().build(portable_config(), masked, B200)
    assert plan.describe()["valid_token_mask"] == "direct_key_mask"
    paired = ConfigSpec(
        program=default_program(),
        schedule=replace(
            default_schedule(), attention_launch=Sm100AttentionParams(block_m=256, block_n=128, kv_stages=3)
        ),
    )
    assert PlanBuilder().evaluate(paired, _context(), B200).accepted
    result = PlanBuilder().evaluate(paired, masked, B200)
    assert "mask_not_supported" in _codes(result)
    persistent = ConfigSpec(
        program=default_program(),
        schedule=replace(
            default_schedule(), attention_launch=Sm100AttentionParams(block_m=256, block_n=64, kv_stages=8)
        ),
    )
    assert PlanBuilder().evaluate(persistent, masked, B200).accepted


def test_runtime_rules() -> None:
    tiled = ConfigSpec(
        program=default_program(),
        schedule=default_schedule(RuntimeBackend.BATCH_TILED_CUDA_GRAPH, batch_tile_size=2),
    )
    assert "tile_not_smaller_than_batch" in _codes(PlanBuilder().evaluate(tiled, _context(), B200))
    plan = PlanBuilder().build(tiled, _context(batch_size=8), B200)
    assert plan.inner_context.batch_size == 2 and plan.outer_context.batch_size == 8

    streamed = portable_streamed_config(microbatch_size=3)
    assert "microbatch_not_divisor" in _codes(PlanBuilder().evaluate(streamed, _context(batch_size=8), B200))
    assert "microbatch_exceeds_batch" in _codes(PlanBuilder().evaluate(streamed, _context(batch_size=2), B200))
    plan = PlanBuilder().build(portable_streamed_config(microbatch_size=2), _context(batch_size=8), B200)
    assert plan.use_streamed_execution and plan.inner_context.batch_size == 2


def test_rejection_types() -> None:
    v = ConstraintViolation("c", "f", "m")
    assert v.to_dict() == {"code": "c", "field": "f", "message": "m"}
    with pytest.raises(ValueError):
        CompileRejection("cfg-x", ())
    err = ConfigRejectedError(CompileRejection("cfg-x", (v,)))
    assert "f:c" in str(err)


def test_detect_on_cpu_host_is_not_sm100() -> None:
    caps = HardwareCapabilities.detect(torch.device("cpu"))
    assert caps.device_type == "cpu" and not caps.is_sm100


def test_type_errors() -> None:
    with pytest.raises(TypeError):
        PlanBuilder().evaluate("not a config", _context(), B200)  # type: ignore[arg-type]
    with pytest.raises(TypeError):
        PlanBuilder().evaluate(portable_config(), "ctx", B200)  # type: ignore[arg-type]


# ---------------------------------------------------------------- fused block boundaries


def _fused(fusion: str, **schedule_overrides: object) -> ConfigSpec:
    from solution.config import AttentionBackend

    mma = AttentionBackend.SM100_MMA  # head dims 8..128, as the small official shapes use
    return ConfigSpec(
        program=default_program(attention=mma, fused_boundary=fusion),
        schedule=replace(default_schedule(attention=mma, fused_boundary=fusion), **schedule_overrides),
    )


@pytest.mark.parametrize("fusion", ["linear", "mlp"])
def test_fused_boundaries_drop_the_fused_projections_launch_records(fusion: str) -> None:
    from solution.config import FFNBackend, ResidualNormBackend

    config = _fused(fusion)
    assert config.program.residual_norm is ResidualNormBackend.SM100_LINEAR_MIXED
    assert (config.program.ffn is FFNBackend.SM100_FUSED_MLP_BOUNDARY) == (fusion == "mlp")
    assert config.schedule.attention_output_projection_launch is None
    assert config.schedule.ffn_launch is None
    assert (config.schedule.ffn_input_launch is None) == (fusion == "mlp")
    assert ConfigSpec.from_dict(json.loads(config.canonical_json())) == config
    with pytest.raises(ValueError, match="attention_output_projection_launch"):
        _fused(fusion, attention_output_projection_launch=Sm100GemmParams())
    with pytest.raises(ValueError, match="fused_boundary"):
        default_program(fused_boundary="everything")


@pytest.mark.parametrize("fusion", ["linear", "mlp"])
def test_fused_boundaries_accepted_for_their_built_widths(fusion: str) -> None:
    """Both boundaries are built for d_model 32, 64 and 128; the Linear one
    also for 512, 768 and 1024 (the row-complete tcgen05 GEMM)."""

    for width in (32, 64, 128, 512, 768, 1024):
        heads = max(1, width // 64)
        context = _context(d_model=width, num_heads=heads, ffn_dim=4 * width)
        accepted = PlanBuilder().evaluate(_fused(fusion), context, B200).accepted
        assert accepted == (fusion == "linear" or width <= 128), width
    result = PlanBuilder().evaluate(_fused(fusion), _context(), B200)  # d_model 256
    assert not result.accepted and "unsupported_shape" in _codes(result)
    fields = {v.field for v in result.violations}
    assert "program.residual_norm" in fields
    if fusion == "mlp":
        wide = PlanBuilder().evaluate(_fused(fusion), _context(d_model=1024, num_heads=16, ffn_dim=4096), B200)
        assert {v.field for v in wide.violations} == {"program.ffn"}


def test_fused_mlp_needs_the_fused_linear_boundary_and_ffn_dim_multiple_of_16() -> None:
    from solution.config import FFNBackend

    ok = _fused("mlp")
    assert PlanBuilder().evaluate(ok, _context(d_model=128, ffn_dim=128), B200).accepted
    result = PlanBuilder().evaluate(ok, _context(d_model=128, ffn_dim=136), B200)  # 136 % 16 != 0
    assert not result.accepted and {v.field for v in result.violations} == {"ffn_dim"}
    unfused_norm = ConfigSpec(
        program=replace(default_program(), ffn=FFNBackend.SM100_FUSED_MLP_BOUNDARY),
        schedule=replace(default_schedule(), ffn_input_launch=None),
    )
    result = PlanBuilder().evaluate(unfused_norm, _context(d_model=128, ffn_dim=128), B200)
    assert not result.accepted and "backend_incompatible" in _codes(result)


def test_fused_plan_keeps_the_expected_trace_roles() -> None:
    plan = PlanBuilder().build(_fused("mlp"), _context(d_model=128, ffn_dim=128), B200)
    trace = plan.expected_trace
    assert trace.residual_norm_backend.value == "sm100_linear_mixed"
    assert trace.ffn_backend.value == "sm100_fused_mlp_boundary"
    assert trace.attention_output_projection_calls == trace.ffn_output_projection_calls == 2
    assert trace.residual_norm_calls == 4


def test_official_bench_schedules_are_accepted_for_every_official_shape() -> None:
    """Every schedule `bench.py --workload official` times compiles for its shape."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from workloads import OFFICIAL_SHAPES

    for case, cfg in OFFICIAL_SHAPES.items():
        if case == "official_14":
            continue
        context = _context(
            batch_size=cfg.batch_size, seq_len=cfg.seq_len, d_model=cfg.d_model, num_heads=cfg.num_heads,
            ffn_dim=cfg.ffn_dim, num_layers=cfg.num_layers,
        )
        for eager in (False, True):
            for name, config in bench.official_schedules(cfg, eager):
                result = PlanBuilder().evaluate(config, context, B200)
                assert result.accepted, (case, name, [v.message for v in result.violations])


# ---------------------------------------------------------------- whole-forward runtime
def _sequence_resident() -> ConfigSpec:
    from solution.config import AttentionBackend, RuntimeBackend

    mma = AttentionBackend.SM100_MMA
    return ConfigSpec(
        program=default_program(attention=mma), schedule=default_schedule(RuntimeBackend.SEQUENCE_RESIDENT, attention=mma)
    )


def test_sequence_resident_runtime_accepts_the_small_official_shapes() -> None:
    config = _sequence_resident()
    assert ConfigSpec.from_dict(json.loads(config.canonical_json())) == config
    for heads, seq in ((4, 128), (1, 128), (2, 128), (4, 32), (4, 64)):
        context = _context(d_model=128, num_heads=heads, ffn_dim=128, seq_len=seq, batch_size=64, num_layers=4)
        result = PlanBuilder().evaluate(config, context, B200)
        assert result.accepted, (heads, seq, _codes(result))
        assert result.plan.use_sequence_resident


def test_sequence_resident_runtime_rejects_what_the_kernel_does_not_build() -> None:
    config = _sequence_resident()
    base = dict(d_model=128, num_heads=4, ffn_dim=128, seq_len=128, batch_size=64, num_layers=4)
    cases = [
        (dict(d_model=256, num_heads=4, ffn_dim=1024), "unsupported_shape"),
        (dict(num_heads=16), "unsupported_shape"),
        (dict(seq_len=1024), "unsupported_shape"),
        (dict(num_layers=9), "unsupported_shape"),
        (dict(has_valid_token_mask=True), "mask_not_supported"),
        (dict(dtype=torch.bfloat16), "unsupported_dtype"),
    ]
    for overrides, code in cases:
        result = PlanBuilder().evaluate(config, _context(**{**base, **overrides}), B200)
        assert not result.accepted and code in _codes(result), (overrides, _codes(result))
        assert "schedule.runtime" in {v.field for v in result.violations}
