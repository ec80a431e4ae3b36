"""The CPU oracle against the reference's own outputs (tests/golden/).

The golden fixtures were produced by running the reference's official
``BaselineTransformer`` and its ``solution`` portable program on CPU
(tests/golden/make_golden.py).  These tests pin the numpy restatement and the
seeded weight/input generators to them before anything is compared with the
GPU path.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import load_golden, parity_errors

from oracle import (
    OfficialConfig,
    attention_core,
    attention_reference,
    attention_rows,
    gelu_erf,
    layer_norm,
    official_input,
    official_state_dict,
    transformer_forward,
    transformer_forward_tail,
)
from oracle.weights import per_row_input, state_checksum, state_to_numpy

CASES = ["c1_official", "tiny", "ragged_s300", "noncausal", "masked", "s1"]


def _config(golden: dict[str, np.ndarray]) -> OfficialConfig:
    b, s, d, h, f, layers, causal = (int(v) for v in golden["config"])
    return OfficialConfig(b, s, d, h, f, layers, bool(causal))


@pytest.mark.parametrize("name", CASES)
def test_weights_match_reference_init(name: str) -> None:
    golden = load_golden(name)
    state = official_state_dict(_config(golden), seed=0)
    assert state_checksum(state) == pytest.approx(float(golden["weight_checksum"]), rel=0, abs=1e-9)


@pytest.mark.parametrize("name", CASES)
def test_input_matches_reference_generator(name: str) -> None:
    golden = load_golden(name)
    if float(golden["padding_ratio"]) > 0:
        pytest.skip("padded inputs are stored verbatim")
    x = official_input(_config(golden), int(golden["input_seed"]))
    assert float(x.double().sum()) == pytest.approx(float(golden["input_checksum"]), abs=1e-9)
    assert float(x.double().abs().sum()) == pytest.approx(float(golden["input_abs_checksum"]), abs=1e-9)
    if "input" in golden:
        np.testing.assert_array_equal(x.numpy(), golden["input"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_forward_matches_reference(name: str) -> None:
    golden = load_golden(name)
    cfg = _config(golden)
    state = state_to_numpy(official_state_dict(cfg, seed=0))
    if "input" in golden:
        x = golden["input"]
    else:
        x = official_input(cfg, int(golden["input_seed"])).numpy()
    mask = golden["mask"] if float(golden["padding_ratio"]) > 0 else None
    y = transformer_forward(
        x, state, num_heads=cfg.num_heads, num_layers=cfg.num_layers, causal=cfg.causal, valid_token_mask=mask
    )
    max_abs, rel = parity_errors(y, golden["output"])
    # Same fp32 maths with a different summation order: agreement to ~1e-6.
    assert max_abs < 5e-5, max_abs
    assert rel < 1e-5, rel


def test_reference_solution_matched_official_when_fixtures_were_made() -> None:
    for name in CASES:
        golden = load_golden(name)
        assert float(golden["solution_max_abs_diff"]) == 0.0
        assert float(golden["all_true_mask_max_abs_diff"]) == 0.0


def test_query_block_size_does_not_change_attention() -> None:
    rng = np.random.default_rng(3)
    cfg = OfficialConfig(2, 70, 64, 2, 128, 1)
    state = state_to_numpy(official_state_dict(cfg, seed=0))
    x = rng.standard_normal((2, 70, 64)).astype(np.float32)
    full = attention_reference(x, state, "layers.0.attention", 2, True, query_block=1024)
    blocked = attention_reference(x, state, "layers.0.attention", 2, True, query_block=16)
    np.testing.assert_allclose(blocked, full, rtol=1e-5, atol=1e-6)


def test_oracle_ops_match_torch() -> None:
    rng = np.random.default_rng(4)
    x = rng.standard_normal((5, 96)).astype(np.float32) * 3
    w = rng.standard_normal(96).astype(np.float32)
    b = rng.standard_normal(96).astype(np.float32)
    ref = torch.nn.functional.layer_norm(torch.from_numpy(x), (96,), torch.from_numpy(w), torch.from_numpy(b))
    np.testing.assert_allclose(layer_norm(x, w, b), ref.numpy(), rtol=1e-5, atol=1e-5)
    g = torch.nn.functional.gelu(torch.from_numpy(x), approximate="none").numpy()
    np.testing.assert_allclose(gelu_erf(x), g, rtol=1e-6, atol=1e-6)


def test_causal_prefix_property() -> None:
    """Outputs for tokens [0, T) depend only on inputs [0, T) (used at full sizes)."""

    cfg = OfficialConfig(1, 40, 64, 1, 128, 2)
    state = state_to_numpy(official_state_dict(cfg, seed=0))
    x = official_input(cfg, 11).numpy()
    full = transformer_forward(x, state, num_heads=1, num_layers=2)
    prefix = transformer_forward(x[:, :17], state, num_heads=1, num_layers=2)
    np.testing.assert_allclose(prefix, full[:, :17], rtol=1e-5, atol=1e-5)


def test_batch_row_independence() -> None:
    cfg = OfficialConfig(3, 24, 64, 1, 128, 1)
    state = state_to_numpy(official_state_dict(cfg, seed=0))
    x = official_input(cfg, 12).numpy()
    full = transformer_forward(x, state, num_heads=1, num_layers=1)
    for row in range(3):
        single = transformer_forward(x[row : row + 1], state, num_heads=1, num_layers=1)
        np.testing.assert_allclose(single, full[row : row + 1], rtol=1e-5, atol=1e-5)


def test_per_row_seeds_are_distinct() -> None:
    cfg = OfficialConfig(2, 8, 16, 1, 32, 1)
    a = per_row_input(cfg, 4, 0)
    b = per_row_input(cfg, 4, 1)
    assert a.shape == (1, 8, 16)
    assert not torch.equal(a, b)
    assert torch.equal(a, official_input(OfficialConfig(1, 8, 16, 1, 32, 1), 4))


@pytest.mark.parametrize("causal", [True, False])
def test_attention_rows_equal_the_blocked_core(causal: bool) -> None:
    """The selected-rows attention used by the long-context GPU tests gives the
    rows of the query-blocked core (same op order; BLAS order only)."""

    rng = np.random.default_rng(3)
    q, k, v = rng.standard_normal((3, 1, 1, 700, 64)).astype(np.float32)
    rows = np.array([0, 1, 127, 128, 511, 512, 699])
    full = attention_core(q, k, v, causal)[0, 0, rows]
    got = attention_rows(q[0, 0, rows], k[0, 0], v[0, 0], rows, causal=causal)
    assert np.abs(full - got).max() < 1e-6


def test_tail_forward_equals_the_full_forward_tail() -> None:
    """transformer_forward_tail (every position of the first layers, the tail
    rows of the last) reproduces the last rows of the whole-row oracle."""

    cfg = OfficialConfig(1, 700, 256, 4, 1024, 2, True)
    state = state_to_numpy(official_state_dict(cfg, seed=0))
    x = official_input(cfg, 5).numpy()
    full = transformer_forward(x, state, num_heads=4, num_layers=2)
    tail = transformer_forward_tail(x, state, num_heads=4, num_layers=2, tail=130)
    assert np.abs(full[0, -130:] - tail).max() < 1e-5
