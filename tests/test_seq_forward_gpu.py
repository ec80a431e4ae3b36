"""The whole-forward kernel (b200tx_sequence_forward) against the oracle.

The kernel runs every layer of a d_model = ffn_dim = 128 model in one launch,
one CTA per 128 rows of whole sequences.  Checked here:
* the reference's small official shapes it is built for (official_01/02: four
  heads of 32; official_09: one head of 128; official_10: two heads of 64;
  official_12: sequences of 32 tokens, four per tile) against the oracle
  (the reference forward restated) within the north-star gate;
* a ragged last tile (3 sequences of 64 tokens: 192 rows) and more tiles than
  SMs (the persistent tile loop), against the unfused GPU program;
* repeated calls give identical bits, and the device error word stays clear.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch
from conftest import MAX_ABS_TOL, REL_L2_TOL, parity_errors

from oracle import OfficialConfig, official_input, official_state_dict, transformer_forward
from oracle.weights import state_to_numpy
from solution import _native
from solution.runtimes.sequence_resident import SequenceResidentForward, sequence_resident_supported
from solution.transformer import UserOptimizedTransformer, copy_model_weights

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _clean_error_word():
    _native.device_error(clear=True)
    yield
    assert _native.device_error(clear=True) == 0, "a kernel wait timed out"


def _model(cfg: OfficialConfig) -> UserOptimizedTransformer:
    model = UserOptimizedTransformer(SimpleNamespace(**cfg.__dict__))
    copy_model_weights(official_state_dict(cfg, seed=0), model)
    return model.to(DEV).eval()


def _oracle_rows(cfg: OfficialConfig, x: torch.Tensor, rows: list[int]) -> np.ndarray:
    state = state_to_numpy(official_state_dict(cfg, seed=0))
    return transformer_forward(x[rows].numpy(), state, num_heads=cfg.num_heads, num_layers=cfg.num_layers, causal=True)


@pytest.mark.parametrize(
    "cfg",
    [
        OfficialConfig(1, 128, 128, 4, 128, 4),   # official_02
        OfficialConfig(64, 128, 128, 4, 128, 4),  # official_01
        OfficialConfig(64, 128, 128, 1, 128, 4),  # official_09
        OfficialConfig(64, 128, 128, 2, 128, 4),  # official_10
        OfficialConfig(64, 32, 128, 4, 128, 4),   # official_12
    ],
    ids=["official_02", "official_01", "official_09", "official_10", "official_12"],
)
def test_whole_forward_matches_the_oracle(cfg: OfficialConfig) -> None:
    assert sequence_resident_supported(
        d_model=cfg.d_model, ffn_dim=cfg.ffn_dim, num_heads=cfg.num_heads, seq_len=cfg.seq_len,
        num_layers=cfg.num_layers, causal=True,
    ) is None
    x = official_input(cfg, 11)
    model = _model(cfg)
    runner = SequenceResidentForward(model)
    with torch.inference_mode():
        y = runner(x.to(DEV))
        y2 = runner(x.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "repeated calls must give the same bits"
    rows = sorted({0, cfg.batch_size // 2, cfg.batch_size - 1})
    got = y[rows].float().cpu().numpy()
    assert np.isfinite(got).all()
    max_abs, rel = parity_errors(got, _oracle_rows(cfg, x, rows))
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (max_abs, rel)


@pytest.mark.parametrize(
    "cfg",
    [OfficialConfig(3, 64, 128, 4, 128, 2), OfficialConfig(300, 128, 128, 2, 128, 3)],
    ids=["ragged_last_tile", "more_tiles_than_sms"],
)
def test_whole_forward_matches_the_unfused_program(cfg: OfficialConfig) -> None:
    x = official_input(cfg, 12).to(DEV)
    model = _model(cfg)
    runner = SequenceResidentForward(model)
    with torch.inference_mode():
        y = runner(x)
        ref = model(x)
    torch.cuda.synchronize()
    max_abs, rel = parity_errors(y.float().cpu().numpy(), ref.float().cpu().numpy())
    assert max_abs < 2e-2 and rel < 5e-3, (max_abs, rel)
    rows = [0, cfg.batch_size - 1]
    max_abs, rel = parity_errors(y[rows].float().cpu().numpy(), _oracle_rows(cfg, x.cpu(), rows))
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (max_abs, rel)


def test_ineligible_shapes_are_named() -> None:
    why = sequence_resident_supported(d_model=256, ffn_dim=1024, num_heads=4, seq_len=128, num_layers=2, causal=True)
    assert why is not None and "d_model" in why
    assert "heads" in sequence_resident_supported(
        d_model=128, ffn_dim=128, num_heads=16, seq_len=128, num_layers=4, causal=True
    )
    assert "tokens" in sequence_resident_supported(
        d_model=128, ffn_dim=128, num_heads=4, seq_len=1024, num_layers=4, causal=True
    )


@pytest.mark.parametrize(
    "cfg", [OfficialConfig(64, 128, 128, 4, 128, 4), OfficialConfig(64, 32, 128, 2, 128, 2)], ids=["h4_s128", "h2_s32"]
)
def test_model_runs_the_whole_forward_runtime(cfg: OfficialConfig) -> None:
    """UserOptimizedTransformer configured with the sm100_sequence_resident
    runtime: the oracle's output, one kernel observed, the runner rebuilt
    after a weight load."""

    from solution.config import AttentionBackend, ConfigSpec, RuntimeBackend, default_program, default_schedule

    mma = AttentionBackend.SM100_MMA
    model = _model(cfg)
    model.configure_execution(
        config=ConfigSpec(
            program=default_program(attention=mma),
            schedule=default_schedule(RuntimeBackend.SEQUENCE_RESIDENT, attention=mma),
        )
    )
    model.set_execution_observation(True)
    x = official_input(cfg, 13)
    with torch.inference_mode():
        y = model(x.to(DEV))
    torch.cuda.synchronize()
    observed = model.describe_execution_path()["observed_execution_signature"]
    assert observed["runtime_backend"] == "sm100_sequence_resident" and observed["runtime_calls"] == 1
    rows = [0, cfg.batch_size - 1]
    max_abs, rel = parity_errors(y[rows].float().cpu().numpy(), _oracle_rows(cfg, x, rows))
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (max_abs, rel)
    # A weight load invalidates the runner's weight images: zeroed weights must change the output.
    state = {k: torch.zeros_like(v) if k.endswith("ffn_out.weight") else v for k, v in model.state_dict().items()}
    model.load_state_dict(state)
    with torch.inference_mode():
        y_zero = model(x.to(DEV))
    torch.cuda.synchronize()
    assert not torch.equal(y_zero, y)
