"""The sm100 program search space (autotune.search_space) and its GPU sweep.

CPU tests check the space against the plan builder the reference's autotune
loop uses (reference autotune/search_space.py:1589-1693): every branch has an
accepted witness, config_at/index_for are inverse, every enumerated config
round-trips through ConfigSpec JSON, the portable branch is always present,
and a masked context keeps only the attention variants that read masks.  The GPU test
sweeps a small shape exhaustively and checks that every candidate matches
the portable program and that the winner publishes into a registry file the
model then resolves.
"""

from __future__ import annotations

import random
from types import SimpleNamespace

import pytest
import torch

from autotune.search_space import ProgramSearchSpace, SearchContext, StructureSpec
from solution.config import SM100_ATTENTION_VARIANTS, ConfigSpec, RuntimeBackend, portable_config
from solution.plan import ExecutionContext
from solution.plan_builder import HardwareCapabilities, PlanBuilder

B200 = HardwareCapabilities.sm100()


def _context(**overrides: object) -> ExecutionContext:
    base = dict(
        batch_size=4,
        seq_len=256,
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


def _space(scope: str = "resident", max_branches: int | None = None, **overrides: object) -> ProgramSearchSpace:
    extra = {} if max_branches is None else {"max_branches": max_branches}
    return ProgramSearchSpace(
        plan_builder=PlanBuilder(), context=SearchContext(_context(**overrides), scope, B200), **extra
    )


def test_resident_space_has_every_structure_and_the_portable_branch() -> None:
    space = _space()
    runtimes = {b.structure.runtime for b in space.branches}
    assert runtimes == {RuntimeBackend.EAGER, RuntimeBackend.CUDA_GRAPH, RuntimeBackend.BATCH_TILED_CUDA_GRAPH}
    # three attention backends (head_dim 64 has all three) x two precision plans x three
    # runtimes = 18 feasible structures, seeded sample capped at the branch limit
    from autotune.search_space import DEFAULT_MAX_STRUCTURE_BRANCHES

    assert len(space.branches) == DEFAULT_MAX_STRUCTURE_BRANCHES == 16
    portable = space.branch_for(portable_config())
    assert portable is not None and portable.structure.portable
    assert portable.branch_id in space.mandatory_branch_ids
    # every attention variant x 3^4 GEMM variants
    assert portable.cardinality == len(SM100_ATTENTION_VARIANTS) * 81
    assert space.cardinality == sum(b.cardinality for b in space.branches)


def test_index_and_config_are_inverse_and_round_trip_json() -> None:
    space = _space()
    for branch in space.branches:
        for index in range(branch.cardinality):
            config = branch.config_at(index)
            assert branch.index_for(config) == index
            again = ConfigSpec.from_dict(config.to_dict())
            assert again == config and again.config_id == config.config_id
            assert space.branch_for(config) is branch


def test_every_enumerated_config_is_accepted_and_distinct() -> None:
    space = _space()
    configs = list(space.configs())
    assert len(configs) == space.cardinality
    assert len({c.config_id for c in configs}) == len(configs)
    builder = PlanBuilder()
    for config in random.Random(0).sample(configs, 40):
        assert builder.evaluate(config, _context(), B200).accepted


def test_witness_is_accepted_and_default_is_the_portable_config() -> None:
    space = _space()
    portable = space.branch_for(portable_config())
    assert portable.default_config() == portable_config()
    for branch in space.branches:
        assert space.accepted(branch.default_config())


def test_streamed_scope_offers_microbatches() -> None:
    space = _space("streamed", batch_size=8)
    assert {b.structure.runtime for b in space.branches} == {RuntimeBackend.STREAMED}
    branch = space.branches[0]
    micro = next(d for d in branch.domains if d.name == "microbatch_size")
    assert micro.choices == (1, 2, 4, 8)


def test_masked_context_keeps_only_the_mask_reading_attention() -> None:
    space = _space(has_valid_token_mask=True)
    tiles = {branch.parameters_for(c).get("attention_tile") for branch in space.branches for c in branch.configs()
             if space.accepted(c)}
    # the quad, persistent and duo kernels, or the CUDA-core kernel (no tile)
    assert tiles == {"512x64x6", "256x64x8", "256x64x4", "256x128x4", None}


def test_other_head_dims_search_the_warp_mma_and_cuda_core_attention() -> None:
    from solution.config import AttentionBackend

    space = _space(d_model=128, num_heads=4)  # head_dim 32, as the reference's official shapes
    assert {b.structure.attention for b in space.branches} == {
        AttentionBackend.SM100_MMA,
        AttentionBackend.SM100_SIMT,
    }
    assert portable_config(head_dim=32) in list(space.configs())
    assert portable_config(head_dim=32).program.attention is AttentionBackend.SM100_MMA
    space = _space(d_model=1024, num_heads=4)  # head_dim 256: the CUDA-core kernel only
    assert {b.structure.attention for b in space.branches} == {AttentionBackend.SM100_SIMT}


def test_trial_suggestion_and_structure_from_config() -> None:
    class Trial:
        def __init__(self) -> None:
            self.rng = random.Random(3)

        def suggest_categorical(self, name, choices):  # noqa: ANN001, ANN201
            return self.rng.choice(list(choices))

    space = _space()
    for branch in space.branches:
        config = branch.suggest(Trial())
        assert StructureSpec.from_config(config) == branch.structure
        assert branch.index_for(config) is not None


def test_arguments_are_checked() -> None:
    with pytest.raises(ValueError):
        SearchContext(_context(), "other")
    with pytest.raises(ValueError):
        ProgramSearchSpace(plan_builder=PlanBuilder(), context=SearchContext(_context(), "resident", B200),
                           max_branches=0)
    with pytest.raises(ValueError):
        ProgramSearchSpace(
            plan_builder=PlanBuilder(),
            context=SearchContext(_context(device=torch.device("cpu")), "resident",
                                  HardwareCapabilities("cpu", None, None, None, True)),
        )
    space = _space()
    with pytest.raises(IndexError):
        space.branches[0].config_at(space.branches[0].cardinality)


@pytest.mark.gpu
def test_sweep_times_every_candidate_and_publishes_the_winner(tmp_path) -> None:  # noqa: ANN001
    from autotune.sweep import publish_best, sweep
    from deployment.registry import resolve_deployed_config
    from oracle import OfficialConfig, official_input, official_state_dict
    from solution.transformer import UserOptimizedTransformer, copy_model_weights

    cfg = OfficialConfig(4, 256, 256, 4, 1024, 2)
    model = UserOptimizedTransformer(SimpleNamespace(**cfg.__dict__))
    copy_model_weights(official_state_dict(cfg, seed=0), model)
    model = model.to("cuda:0").eval()
    x = official_input(cfg, 2).to("cuda:0")
    with torch.inference_mode():  # the tuned forward runs under inference mode
        context = model._execution_context(x)
    space = ProgramSearchSpace(
        plan_builder=PlanBuilder(), context=SearchContext(context, "resident", HardwareCapabilities.detect(x.device))
    )
    portable = space.branch_for(portable_config())
    results = sweep(model, x, space, warmup=1, repeats=2, limit=portable.cardinality)
    assert len(results) == portable.cardinality  # every candidate within tolerance
    assert all(r.median_ms > 0 for r in results)
    assert results == sorted(results, key=lambda r: r.median_ms)
    target = tmp_path / "deployed.json"
    publish_best(model, x, results, path=target)
    from deployment.environment import EnvironmentFingerprint
    from deployment.registry import ShapeFingerprint

    shape = ShapeFingerprint(4, 256, 4, 256, 2, True, 1024, "float32", 0.0, 1.0)
    resolved = resolve_deployed_config(hardware=EnvironmentFingerprint.detect(x.device), shape=shape, path=target)
    assert resolved == results[0].config


def test_small_d_model_searches_the_fused_boundaries() -> None:
    space = _space(d_model=128, num_heads=2, ffn_dim=128, max_branches=64)  # official_10: head_dim 64
    boundaries = {b.structure.boundary for b in space.branches}
    assert boundaries == {None, "linear", "mlp"}
    for branch in space.branches:
        if branch.structure.boundary is None:
            continue
        config = branch.default_config()
        assert space.accepted(config)
        assert branch.index_for(config) is not None
        assert space.branch_for(config) is branch
        # the fused projections have no GEMM tile parameter
        assert "attention_output_projection_tile" not in branch.parameter_names
        assert ("ffn_input_tile" in branch.parameter_names) == (branch.structure.boundary == "linear")
    # d_model 256 builds no fused boundary
    assert {b.structure.boundary for b in _space(max_branches=64).branches} == {None}


def test_small_official_shapes_search_the_whole_forward_kernel() -> None:
    space = _space(d_model=128, num_heads=4, ffn_dim=128, seq_len=128, batch_size=64, num_layers=4, max_branches=256)
    whole = [b for b in space.branches if b.structure.runtime is RuntimeBackend.SEQUENCE_RESIDENT]
    assert len(whole) == 1
    branch = whole[0]
    assert branch.parameter_names == ()  # one kernel: nothing per launch to tune
    config = branch.default_config()
    assert space.accepted(config)
    assert space.branch_for(config) is branch
    # d_model 256 (the default context here) builds no whole-forward branch
    assert RuntimeBackend.SEQUENCE_RESIDENT not in {b.structure.runtime for b in _space(max_branches=256).branches}
