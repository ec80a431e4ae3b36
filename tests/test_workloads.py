"""The benchmarks' seeded workloads (package ``workloads``) against the
checker's independent generator (``oracle.weights``), which tests/test_oracle.py
pins to checksums of the reference's own state dict: same weights and inputs,
bit for bit."""

from __future__ import annotations

import pytest
import torch

from oracle import OfficialConfig, official_input, official_state_dict
from oracle.weights import per_row_input
from workloads import (
    OFFICIAL_SHAPES,
    REFERENCE_PUBLISHED_MS,
    WorkloadConfig,
    seeded_input,
    seeded_row,
    seeded_state_dict,
)


@pytest.mark.parametrize(
    "cfg",
    [
        WorkloadConfig(2, 128, 256, 4, 1024, 2),
        WorkloadConfig(1, 16, 64, 2, 96, 3, causal=False),
        OFFICIAL_SHAPES["official_07"],
    ],
)
def test_weights_and_inputs_match_the_checker_bit_for_bit(cfg: WorkloadConfig) -> None:
    ours = seeded_state_dict(cfg, seed=0)
    theirs = official_state_dict(OfficialConfig(**cfg.as_dict()), seed=0)
    assert list(ours) == list(theirs)
    for key in ours:
        assert torch.equal(ours[key], theirs[key]), key
    assert torch.equal(seeded_input(cfg, 3), official_input(OfficialConfig(**cfg.as_dict()), 3))
    assert torch.equal(seeded_row(cfg, 4, 2), per_row_input(OfficialConfig(**cfg.as_dict()), 4, 2))


def test_global_rng_state_is_restored() -> None:
    before = torch.get_rng_state()
    seeded_state_dict(WorkloadConfig(1, 8, 64, 2, 64, 1), seed=5)
    assert torch.equal(torch.get_rng_state(), before)


def test_official_shapes_table() -> None:
    assert sorted(OFFICIAL_SHAPES) == [f"official_{i:02d}" for i in range(1, 15)]
    assert set(REFERENCE_PUBLISHED_MS) == set(OFFICIAL_SHAPES)
    for cfg in OFFICIAL_SHAPES.values():
        assert cfg.d_model % cfg.num_heads == 0 and cfg.causal
    assert OFFICIAL_SHAPES["official_14"] == WorkloadConfig(32, 100000, 1024, 16, 1024, 2)
