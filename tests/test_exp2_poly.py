"""The FMA-pipe exp2 that the quad attention kernel uses for part of its softmax.

``exp2_poly_f32x2`` (csrc/sm100_common.cuh) replaces MUFU ex2 for a fixed share
of the score pairs.  These CPU tests restate its steps in numpy float32 with the
coefficients read from the header, and check the properties the kernel relies
on: relative error far below the bf16 rounding of P, an exact zero for masked
(-inf) and very negative inputs, and non-negative finite results everywhere the
softmax can call it (x <= 8).  The GPU attention tests then check the kernel
variants that use it against the fp32 reference.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

HEADER = (
    Path(__file__).resolve().parents[1]
    / "ml-guided-program-search-for-shape-specialized-transformer-optimization_b200"
    / "csrc"
    / "sm100_common.cuh"
)


def _coefficients() -> tuple[np.float32, np.float32, np.float32]:
    text = HEADER.read_text()
    values = {}
    for name in ("kC1", "kC2", "kC3"):
        match = re.search(rf"constexpr float {name} = ([0-9.eE+-]+)f;", text)
        assert match, name
        values[name] = np.float32(float(match.group(1)))
    return values["kC1"], values["kC2"], values["kC3"]


def _fma32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    # float32 x float32 is exact in float64; one rounding of the sum to float32
    # matches a fused multiply-add except in rare double-rounding ties.
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x: np.ndarray) -> np.ndarray:
    """numpy restatement of exp2_poly_f32x2, one lane at a time."""

    c1, c2, c3 = _coefficients()
    magic = np.float32(12582912.0)
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-127.0))
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = _fma32(np.full_like(f, c3), f, np.full_like(f, c2))
    p = _fma32(p, f, np.full_like(f, c1))
    p = _fma32(p, f, np.ones_like(f))
    bits = (t.view(np.uint32).astype(np.uint64) * (1 << 23) + p.view(np.uint32).astype(np.uint64)) % (1 << 32)
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_is_far_below_bf16_rounding() -> None:
    x = np.linspace(-120.0, 8.0, 400_001, dtype=np.float32)
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 2e-4, rel.max()  # bf16 half-ulp is 2e-3


def test_masked_and_tiny_inputs_give_zero_or_tiny_non_negative() -> None:
    assert exp2_poly(np.array([-np.inf], dtype=np.float32))[0] == 0.0
    assert exp2_poly(np.array([-127.0], dtype=np.float32))[0] == 0.0
    assert exp2_poly(np.array([-1e30], dtype=np.float32))[0] == 0.0
    x = np.linspace(-127.0, -110.0, 20_001, dtype=np.float32)
    got = exp2_poly(x)
    assert np.isfinite(got).all() and (got >= 0).all()
    assert (got <= np.float32(2.0**-109)).all()


def test_integer_inputs_are_exact_powers_of_two() -> None:
    x = np.arange(-126, 9, dtype=np.float32)
    np.testing.assert_array_equal(exp2_poly(x), np.exp2(x.astype(np.float64)).astype(np.float32))


def test_softmax_built_on_it_matches_exact_softmax() -> None:
    rng = np.random.default_rng(0)
    s = rng.normal(size=(64, 128)).astype(np.float32) * 3
    m = s.max(axis=1, keepdims=True)
    p = exp2_poly((s - m).astype(np.float32)).astype(np.float64)
    exact = np.exp2((s - m).astype(np.float64))
    np.testing.assert_allclose(p / p.sum(1, keepdims=True), exact / exact.sum(1, keepdims=True), rtol=3e-4)
