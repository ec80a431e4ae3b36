"""Long-context parity past the prefix: the last query tiles at full length.

The prefix tests of test_model_gpu.py check C4 (S = 16 384) and C5
(S = 100 000) on their first 1024 positions, where each query row sees at most
16 KV tiles.  These tests check the rows at the END of those sequences, whose
online softmax runs over 256 (C4) and 1563 (C5) KV tiles with its running max
moved many times, through the same tensor maps, ring slots and 64-bit output
offsets as the full-size runs:

* kernel level, every tensor-core attention variant at the real geometries
  (C4: B2 S16384 H32; C5: one B=1 row, S100000 H16), against
  ``oracle.attention_rows`` for selected (batch, head) pairs: the last 128
  rows, and rows around the 2^13 / 2^16 position boundaries;
* model level, a whole C4 row (B1 of the seed-3 input) through
  ``UserOptimizedTransformer``, whose last 128 positions are compared with
  ``oracle.transformer_forward_tail`` (the reference forward restated; it runs
  every position of layer 0 and the tail of layer 1 on the host).

The reference checks its streamed path the same way, on a whole B=1 row
against its portable forward (benchmarking/shape14_measure.py:139-163).
Tolerances: the attention gate of test_kernels_gpu.py (bf16 P, rel-L2 1e-2,
max-abs 2e-2) and the model gate of the north star (max-abs 2e-2, rel-L2 1e-2).
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch
from conftest import MAX_ABS_TOL, REL_L2_TOL, parity_errors

from oracle import OfficialConfig, attention_rows, official_input, official_state_dict, transformer_forward_tail
from oracle.weights import state_to_numpy
from solution import _native
from solution.kernels import sm100_flash_attention
from solution.transformer import UserOptimizedTransformer, copy_model_weights

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
VARIANTS = [
    _native.ATTN_PINGPONG,
    _native.ATTN_QUAD,
    _native.ATTN_DUO,
    _native.ATTN_PERSISTENT,
    _native.ATTN_PAIRED,
    _native.ATTN_SINGLE,
]


@pytest.fixture(autouse=True)
def _clean_error_word():
    _native.device_error(clear=True)
    yield
    assert _native.device_error(clear=True) == 0, "a kernel wait timed out"


def _drifting_qkv(batch: int, seq: int, heads: int, seed: int) -> torch.Tensor:
    """Packed [B, S, 3*H*64] bf16 q/k/v whose key norms grow along the
    sequence (x1 -> x3), so each late query row's running max keeps moving,
    and whose values carry a position-dependent offset, so a dropped or
    doubly counted early KV tile shows in the output."""

    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(batch, seq, 3, heads, 64, generator=g)
    pos = torch.arange(seq, dtype=torch.float32)
    qkv[:, :, 1] *= (1.0 + 2.0 * pos / seq)[None, :, None, None]
    qkv[:, :, 2] += torch.sin(pos / 977.0)[None, :, None, None]
    return qkv.reshape(batch, seq, 3 * heads * 64).to(torch.bfloat16)


def _check_rows(qkv: torch.Tensor, out: torch.Tensor, heads: int, picks: list[tuple[int, int]], rows: np.ndarray) -> None:
    batch, seq, _ = qkv.shape
    d_model = heads * 64
    got = out.float().cpu().view(batch, seq, heads, 64)
    for b, h in picks:
        q = qkv[b, rows, h * 64:(h + 1) * 64].float().numpy()
        k = qkv[b, :, d_model + h * 64:d_model + (h + 1) * 64].float().numpy()
        v = qkv[b, :, 2 * d_model + h * 64:2 * d_model + (h + 1) * 64].float().numpy()
        ref = attention_rows(q, k, v, rows, causal=True)
        max_abs, rel = parity_errors(got[b, rows, h].numpy(), ref)
        assert np.isfinite(got[b, rows, h].numpy()).all()
        assert rel < 1e-2 and max_abs < 2e-2, (b, h, max_abs, rel)


@pytest.fixture(scope="module")
def c4_qkv() -> torch.Tensor:
    return _drifting_qkv(2, 16384, 32, seed=4)


@pytest.fixture(scope="module")
def c5_qkv() -> torch.Tensor:
    return _drifting_qkv(1, 100000, 16, seed=5)


@pytest.mark.parametrize("variant", VARIANTS)
def test_attention_tail_rows_at_c4_geometry(c4_qkv: torch.Tensor, variant: int) -> None:
    """C4 geometry (S16384, 32 heads, D2048; two batch rows for the batch
    stride): rows 16256-16383 and 8190-8193 of (b0, h0), (b1, h31), (b1, h7)."""

    with torch.inference_mode():
        out, _ = sm100_flash_attention(c4_qkv.to(DEV), 32, causal=True, variant=variant)
    torch.cuda.synchronize()
    rows = np.concatenate([np.arange(8190, 8194), np.arange(16256, 16384)])
    _check_rows(c4_qkv, out, 32, [(0, 0), (1, 31), (1, 7)], rows)


@pytest.mark.parametrize("variant", VARIANTS)
def test_attention_tail_rows_at_c5_geometry(c5_qkv: torch.Tensor, variant: int) -> None:
    """One C5 row (S100000, 16 heads, D1024): rows 99872-99999, 65534-65537
    (past 2^16) and 0-1 of heads 0 and 15."""

    with torch.inference_mode():
        out, _ = sm100_flash_attention(c5_qkv.to(DEV), 16, causal=True, variant=variant)
    torch.cuda.synchronize()
    rows = np.concatenate([np.arange(2), np.arange(65534, 65538), np.arange(99872, 100000)])
    _check_rows(c5_qkv, out, 16, [(0, 0), (0, 15)], rows)


def test_model_c4_row_tail() -> None:
    """One C4 row (seed 3, row 0; S16384 D2048 H32 F8192 L2) through the whole
    model: its last 128 positions against the reference forward restated."""

    cfg = OfficialConfig(4, 16384, 2048, 32, 8192, 2, True)
    state = official_state_dict(cfg, seed=0)
    x = official_input(cfg, 3, batch_rows=slice(0, 1))
    model = UserOptimizedTransformer(SimpleNamespace(**{**cfg.__dict__, "batch_size": 1}))
    copy_model_weights(state, model)
    model = model.to(DEV).eval()
    with torch.inference_mode():
        y = model(x.to(DEV))
    torch.cuda.synchronize()
    got = y[0, -128:].float().cpu().numpy()
    ref = transformer_forward_tail(
        x.numpy(), state_to_numpy(state), num_heads=cfg.num_heads, num_layers=cfg.num_layers, tail=128
    )
    assert np.isfinite(got).all()
    max_abs, rel = parity_errors(got, ref)
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (max_abs, rel)
