"""Kernel-level parity: each libb200tx kernel, called through the C ABI, against
the CPU oracle on the same seeded inputs, including ragged and tiny edge cases.

Tolerances: the fp32 residual sum is exact; fp32 outputs agree to fp32
rounding; bf16 outputs carry one bf16 rounding (relative 2^-9), so they are
checked at rel-L2 <= 4e-3; attention rounds P to bf16 before P.V (as the
reference casts probabilities to the activation dtype), checked at
rel-L2 <= 1e-2 and max-abs <= 2e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import parity_errors

from oracle import attention_core, gelu_erf, layer_norm
from solution import _native
from solution.kernels import (
    sm100_flash_attention,
    sm100_initial_layer_norm,
    sm100_linear,
    sm100_residual_layer_norm,
)

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _clean_error_word():
    _native.device_error(clear=True)
    yield
    assert _native.device_error(clear=True) == 0, "a kernel wait timed out"


@pytest.mark.parametrize(
    ("rows", "cols", "update_dtype", "in_dtype"),
    [
        (1, 128, torch.bfloat16, torch.float32),
        (7, 256, torch.bfloat16, torch.float32),
        (1000, 768, torch.bfloat16, torch.float32),
        (513, 1024, torch.float32, torch.float32),
        (64, 2048, torch.bfloat16, torch.float32),
        (33, 4096, torch.bfloat16, torch.float32),
        (17, 96, torch.bfloat16, torch.float32),  # generic path (cols % 128 != 0)
        (9, 4104, torch.float32, torch.float32),  # generic path, wide
        (40, 1024, torch.bfloat16, torch.bfloat16),  # bf16 residual input
    ],
)
def test_residual_layer_norm(rows: int, cols: int, update_dtype: torch.dtype, in_dtype: torch.dtype) -> None:
    g = torch.Generator().manual_seed(rows * 31 + cols)
    resid = (torch.randn(rows, cols, generator=g) * 2).to(in_dtype)
    update = torch.randn(rows, cols, generator=g).to(update_dtype)
    norm = torch.nn.LayerNorm(cols)
    with torch.no_grad():
        norm.weight.copy_(torch.randn(cols, generator=g))
        norm.bias.copy_(torch.randn(cols, generator=g))
    norm = norm.to(DEV)
    ref_r = resid.float().numpy() + update.float().numpy()
    ref_n = layer_norm(ref_r, norm.weight.detach().cpu().numpy(), norm.bias.detach().cpu().numpy())
    with torch.inference_mode():
        r, n, marker = sm100_residual_layer_norm(resid.to(DEV), update.to(DEV), norm, final_boundary=False)
        _, n32, _ = sm100_residual_layer_norm(resid.to(DEV), update.to(DEV), norm, final_boundary=True)
    torch.cuda.synchronize()
    assert marker == "sm100_residual_layer_norm"
    np.testing.assert_array_equal(r.cpu().numpy(), ref_r.astype(np.float32))
    max_abs, rel = parity_errors(_bf16_np(n), ref_n)
    assert rel < 4e-3 and max_abs < 6e-2, (max_abs, rel)
    max_abs, rel = parity_errors(n32.cpu().numpy(), ref_n)
    assert max_abs < 2e-4 and rel < 1e-5, (max_abs, rel)


def test_residual_layer_norm_in_place() -> None:
    g = torch.Generator().manual_seed(5)
    resid = torch.randn(300, 1024, generator=g)
    update = torch.randn(300, 1024, generator=g).to(torch.bfloat16)
    norm = torch.nn.LayerNorm(1024).to(DEV)
    expected = resid.numpy() + update.float().numpy()
    stream = resid.to(DEV)
    with torch.inference_mode():
        sm100_residual_layer_norm(stream, update.to(DEV), norm, final_boundary=False, residual_out=stream)
    np.testing.assert_array_equal(stream.cpu().numpy(), expected)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_initial_layer_norm(dtype: torch.dtype) -> None:
    g = torch.Generator().manual_seed(9)
    x = torch.randn(129, 768, generator=g).to(dtype)
    norm = torch.nn.LayerNorm(768).to(DEV)
    ref = layer_norm(x.float().numpy(), np.ones(768, np.float32), np.zeros(768, np.float32))
    with torch.inference_mode():
        n, marker = sm100_initial_layer_norm(x.to(DEV), norm)
    assert marker == "sm100_initial_layer_norm" and n.dtype == torch.bfloat16
    max_abs, rel = parity_errors(_bf16_np(n), ref)
    assert rel < 4e-3 and max_abs < 4e-2


@pytest.mark.parametrize(
    ("m", "n", "k", "gelu", "out_dtype", "bias"),
    [
        (1, 8, 8, False, torch.float32, True),
        (127, 264, 72, True, torch.bfloat16, True),
        (128, 256, 64, False, torch.float32, False),
        (129, 768, 768, True, torch.float32, True),
        (1000, 3072, 1024, False, torch.bfloat16, True),
        (4097, 1024, 4096, False, torch.float32, True),
        (300, 2304, 768, True, torch.bfloat16, True),
        (257, 392, 136, False, torch.bfloat16, True),  # pair tiles: ragged M and N halves
        (16384, 1024, 1024, False, torch.bfloat16, True),  # C2 out-projection shape
    ],
)
@pytest.mark.parametrize("variant", [_native.GEMM_1SM, _native.GEMM_PAIR, _native.GEMM_WARP])
def test_linear(m: int, n: int, k: int, gelu: bool, out_dtype: torch.dtype, bias: bool, variant: int) -> None:
    g = torch.Generator().manual_seed(m + 7 * n + 13 * k)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) / k**0.5).to(torch.bfloat16)
    b = torch.randn(n, generator=g) if bias else None
    ref = a.float().numpy() @ w.float().numpy().T
    if b is not None:
        ref = ref + b.numpy()
    if gelu:
        ref = gelu_erf(ref.astype(np.float32))
    with torch.inference_mode():
        out, marker = sm100_linear(
            a.to(DEV), w.to(DEV), None if b is None else b.to(DEV), gelu=gelu, out_dtype=out_dtype,
            variant=variant,
        )
    torch.cuda.synchronize()
    assert marker == ("sm100_linear_gelu" if gelu else "sm100_linear")
    max_abs, rel = parity_errors(out.float().cpu().numpy(), ref)
    if out_dtype == torch.float32:
        assert rel < 1e-5, rel
    else:
        assert rel < 4e-3, rel


def test_linear_variants_agree_bitwise() -> None:
    """Both GEMM variants accumulate each output in the same K order: equal bits."""

    g = torch.Generator().manual_seed(5)
    a = torch.randn(2000, 1024, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(3072, 1024, generator=g) / 32).to(torch.bfloat16).to(DEV)
    b = torch.randn(3072, generator=g).to(DEV)
    with torch.inference_mode():
        one, _ = sm100_linear(a, w, b, gelu=True, variant=_native.GEMM_1SM)
        two, _ = sm100_linear(a, w, b, gelu=True, variant=_native.GEMM_PAIR)
        again, _ = sm100_linear(a, w, b, gelu=True, variant=_native.GEMM_PAIR)
    assert torch.equal(two, again)
    max_abs, rel = parity_errors(_bf16_np(one), _bf16_np(two))
    assert rel < 1e-3, rel


def test_linear_bias_not_16_byte_aligned() -> None:
    """A bias view one float into its storage takes the per-column load path."""

    g = torch.Generator().manual_seed(4)
    a = torch.randn(300, 512, generator=g).to(torch.bfloat16)
    w = (torch.randn(1024, 512, generator=g) / 16).to(torch.bfloat16)
    storage = torch.randn(1025, generator=g)
    b = storage[1:]
    ref = a.float().numpy() @ w.float().numpy().T + b.numpy()
    with torch.inference_mode():
        bias_dev = storage.to(DEV)[1:]
        assert bias_dev.data_ptr() % 16 != 0
        out, _ = sm100_linear(a.to(DEV), w.to(DEV), bias_dev, out_dtype=torch.float32)
    assert parity_errors(out.cpu().numpy(), ref)[1] < 1e-5


def test_linear_three_dimensional_input() -> None:
    g = torch.Generator().manual_seed(1)
    a = torch.randn(3, 50, 256, generator=g).to(torch.bfloat16)
    w = torch.randn(512, 256, generator=g).to(torch.bfloat16)
    with torch.inference_mode():
        out, _ = sm100_linear(a.to(DEV), w.to(DEV), None, out_dtype=torch.float32)
    ref = a.float().numpy() @ w.float().numpy().T
    assert out.shape == (3, 50, 512)
    assert parity_errors(out.cpu().numpy(), ref)[1] < 1e-5


VARIANTS = [
    _native.ATTN_PAIRED,
    _native.ATTN_SINGLE,
    _native.ATTN_QUAD,
    _native.ATTN_PERSISTENT,
    _native.ATTN_DUO,
    _native.ATTN_PINGPONG,
]
MASKED_VARIANTS = [_native.ATTN_QUAD, _native.ATTN_PERSISTENT, _native.ATTN_DUO, _native.ATTN_PINGPONG]


def _attention_case(batch: int, seq: int, heads: int, causal: bool, seed: int, variant: int) -> None:
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(batch, seq, 3 * heads * 64, generator=g).to(torch.bfloat16)
    q, k, v = qkv.float().view(batch, seq, 3, heads, 64).permute(2, 0, 3, 1, 4).numpy()
    ref = attention_core(q, k, v, causal).transpose(0, 2, 1, 3).reshape(batch, seq, heads * 64)
    with torch.inference_mode():
        out, marker = sm100_flash_attention(qkv.to(DEV), heads, causal=causal, variant=variant)
    torch.cuda.synchronize()
    assert marker == "sm100_flash_attention"
    max_abs, rel = parity_errors(_bf16_np(out), ref)
    assert rel < 1e-2 and max_abs < 2e-2, (batch, seq, heads, causal, variant, max_abs, rel)


@pytest.mark.parametrize(
    ("batch", "seq", "heads", "causal"),
    [
        (1, 1, 1, True),
        (2, 17, 1, True),
        (1, 127, 2, True),
        (1, 128, 1, True),
        (3, 129, 2, True),
        (1, 300, 5, True),
        (2, 1000, 2, True),
        (1, 1, 1, False),
        (2, 200, 2, False),
        (1, 385, 1, False),
        (2, 256, 3, True),  # even number of query tiles
        (1, 384, 2, True),  # odd: the last pair has one tile
        (1, 640, 2, True),  # five query tiles: the last quad has one
        (2, 1500, 1, False),
    ],
)
@pytest.mark.parametrize("variant", VARIANTS)
def test_attention_edges(batch: int, seq: int, heads: int, causal: bool, variant: int) -> None:
    _attention_case(batch, seq, heads, causal, seed=batch * 1000 + seq + heads, variant=variant)


@pytest.mark.parametrize("variant", VARIANTS)
def test_attention_long_sequence(variant: int) -> None:
    """Many KV tiles per query tile (64 on the last), running max moved repeatedly."""

    _attention_case(1, 8192, 2, True, seed=77, variant=variant)


@pytest.mark.parametrize("variant", VARIANTS)
def test_attention_is_deterministic(variant: int) -> None:
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(2, 700, 3 * 4 * 64, generator=g).to(torch.bfloat16).to(DEV)
    with torch.inference_mode():
        a, _ = sm100_flash_attention(qkv, 4, variant=variant)
        b, _ = sm100_flash_attention(qkv, 4, variant=variant)
    assert torch.equal(a, b)


@pytest.mark.parametrize(
    ("batch", "seq", "heads", "causal"), [(8, 1024, 16, True), (4, 640, 40, False), (8, 2048, 8, True), (3, 1000, 20, True)]
)
def test_attention_persistent_many_items_per_cta(batch: int, seq: int, heads: int, causal: bool) -> None:
    """More work items than 2x the SM count: each CTA of the persistent kernel
    walks several items, its barrier phases and Q buffers carried across them."""

    _attention_case(batch, seq, heads, causal, seed=seq + heads, variant=_native.ATTN_PERSISTENT)


@pytest.mark.parametrize(
    ("batch", "seq", "heads", "causal"),
    [(8, 1024, 16, True), (4, 640, 40, False), (8, 2048, 8, True), (3, 1000, 20, True), (1, 4096, 148, True)],
)
def test_attention_pingpong_many_items_per_cta(batch: int, seq: int, heads: int, causal: bool) -> None:
    """More work items than CTAs: each persistent PINGPONG CTA walks several
    items, its Q buffers, K/V ring positions and barrier phases carried across
    them, items of different lengths interleaved by the snake order."""

    _attention_case(batch, seq, heads, causal, seed=seq + 7 * heads, variant=_native.ATTN_PINGPONG)


@pytest.mark.parametrize(
    ("batch", "seq", "heads", "causal"), [(8, 2048, 16, True), (4, 640, 40, False), (16, 512, 12, True)]
)
def test_attention_duo_two_ctas_per_sm(batch: int, seq: int, heads: int, causal: bool) -> None:
    """More CTAs than 2x the SM count: two DUO CTAs share each SM's TMEM and
    shared memory, and CTAs of short and long causal pairs interleave."""

    _attention_case(batch, seq, heads, causal, seed=seq + 3 * heads, variant=_native.ATTN_DUO)


@pytest.mark.parametrize("causal", [True, False])
def test_attention_variants_agree(causal: bool) -> None:
    g = torch.Generator().manual_seed(13)
    qkv = torch.randn(3, 1000, 3 * 2 * 64, generator=g).to(torch.bfloat16).to(DEV)
    with torch.inference_mode():
        a, _ = sm100_flash_attention(qkv, 2, causal=causal, variant=_native.ATTN_PAIRED)
        for other in (_native.ATTN_SINGLE, _native.ATTN_QUAD, _native.ATTN_PERSISTENT, _native.ATTN_DUO,
                      _native.ATTN_PINGPONG):
            b, _ = sm100_flash_attention(qkv, 2, causal=causal, variant=other)
            max_abs, rel = parity_errors(_bf16_np(a), _bf16_np(b))
            # Two bf16 results of different summation orders: a few bf16 ulps apart.
            assert rel < 5e-3 and max_abs < 4e-2, (other, max_abs, rel)


@pytest.mark.parametrize("variant", VARIANTS)
def test_attention_large_logits_stay_finite(variant: int) -> None:
    """Scores of |s| ~ 100 exercise the stale-max threshold and rescaling."""

    g = torch.Generator().manual_seed(8)
    qkv = (torch.randn(1, 512, 3 * 64, generator=g) * 6).to(torch.bfloat16)
    q, k, v = qkv.float().view(1, 512, 3, 1, 64).permute(2, 0, 3, 1, 4).numpy()
    ref = attention_core(q, k, v, True).transpose(0, 2, 1, 3).reshape(1, 512, 64)
    with torch.inference_mode():
        out, _ = sm100_flash_attention(qkv.to(DEV), 1, variant=variant)
    got = _bf16_np(out)
    assert np.isfinite(got).all()
    max_abs, rel = parity_errors(got, ref)
    assert rel < 2e-2, rel


# ---------------------------------------------------------------- padding masks
def _masked_attention_reference(
    q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool, key_valid: np.ndarray
) -> np.ndarray:
    """Official scores with causal and key-padding -inf (official :97-112); a
    query with no valid key gets a zero row (the kernel's convention; the
    reference's NaN row there is zeroed by the caller's masked_fill)."""

    seq = q.shape[2]
    scores = np.matmul(q, k.transpose(0, 1, 3, 2)) * np.float32(q.shape[-1] ** -0.5)
    if causal:
        scores = np.where(np.triu(np.ones((seq, seq), bool), 1)[None, None], np.float32(-np.inf), scores)
    scores = np.where(~key_valid[:, None, None, :], np.float32(-np.inf), scores)
    m = scores.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, np.float32(0.0))
    p = np.exp(scores - m, dtype=np.float32)
    l = p.sum(axis=-1, keepdims=True)
    return np.matmul(p, v) / np.where(l > 0, l, np.float32(1.0))


@pytest.mark.parametrize(
    ("batch", "seq", "heads", "causal", "pattern"),
    [
        (2, 300, 2, True, "random"),
        (2, 640, 1, True, "left"),  # queries before the first valid key see none
        (3, 257, 2, False, "right"),
        (2, 1000, 2, True, "one_empty_row"),
        (1, 129, 1, False, "random"),
        (8, 768, 16, True, "random"),  # several work items per persistent CTA
    ],
)
@pytest.mark.parametrize("variant", MASKED_VARIANTS)
def test_attention_key_padding_mask(
    batch: int, seq: int, heads: int, causal: bool, pattern: str, variant: int
) -> None:
    g = torch.Generator().manual_seed(seq + heads)
    qkv = torch.randn(batch, seq, 3 * heads * 64, generator=g).to(torch.bfloat16)
    if pattern == "random":
        valid = torch.rand(batch, seq, generator=g) > 0.3
    elif pattern == "left":
        valid = torch.arange(seq)[None, :] >= torch.tensor([[70], [200]])[:batch]
    elif pattern == "right":
        valid = torch.arange(seq)[None, :] < torch.tensor([[257], [100], [1]])[:batch]
    else:
        valid = torch.rand(batch, seq, generator=g) > 0.5
        valid[1] = False
    q, k, v = qkv.float().view(batch, seq, 3, heads, 64).permute(2, 0, 3, 1, 4).numpy()
    ref = _masked_attention_reference(q, k, v, causal, valid.numpy())
    ref = ref.transpose(0, 2, 1, 3).reshape(batch, seq, heads * 64)
    key_valid = valid.to(DEV).view(torch.uint8)
    with torch.inference_mode():
        out, _ = sm100_flash_attention(qkv.to(DEV), heads, causal=causal, key_valid=key_valid, variant=variant)
    got = _bf16_np(out)
    assert np.isfinite(got).all()
    max_abs, rel = parity_errors(got, ref)
    assert rel < 1e-2 and max_abs < 2e-2, (pattern, max_abs, rel)
    if pattern == "one_empty_row":
        assert not got[1].any()


@pytest.mark.parametrize("variant", MASKED_VARIANTS)
def test_attention_all_valid_mask_equals_unmasked(variant: int) -> None:
    g = torch.Generator().manual_seed(21)
    qkv = torch.randn(2, 700, 3 * 4 * 64, generator=g).to(torch.bfloat16).to(DEV)
    ones = torch.ones(2, 700, dtype=torch.uint8, device=DEV)
    with torch.inference_mode():
        a, _ = sm100_flash_attention(qkv, 4, variant=variant)
        b, _ = sm100_flash_attention(qkv, 4, key_valid=ones, variant=variant)
    assert torch.equal(a, b)


def test_attention_mask_needs_the_quad_variant() -> None:
    qkv = torch.zeros(1, 128, 3 * 64, dtype=torch.bfloat16, device=DEV)
    ones = torch.ones(1, 128, dtype=torch.uint8, device=DEV)
    with torch.inference_mode(), pytest.raises(ValueError, match="QUAD"):
        sm100_flash_attention(qkv, 1, key_valid=ones, variant=_native.ATTN_PAIRED)


@pytest.mark.parametrize("mode", [1, 2, 4, 2 | 4, 1 | 4])
@pytest.mark.parametrize("cols", [1024, 96])
def test_residual_layer_norm_row_mask(mode: int, cols: int) -> None:
    rows = 300
    g = torch.Generator().manual_seed(mode * 7 + cols)
    resid = torch.randn(rows, cols, generator=g) * 2
    update = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    valid = torch.rand(rows, generator=g) > 0.4
    gamma = torch.randn(cols, generator=g)
    beta = torch.randn(cols, generator=g)
    ln = torch.nn.LayerNorm(cols).to(DEV)
    with torch.no_grad():
        ln.weight.copy_(gamma)
        ln.bias.copy_(beta)
    r = resid + update.float()
    keep = valid[:, None]
    if mode & 1:
        r = torch.where(keep, r, resid)
    if mode & 2:
        r = torch.where(keep, r, torch.zeros(()))
    n = torch.from_numpy(layer_norm(r.numpy(), gamma.numpy(), beta.numpy()))
    if mode & 4:
        n = torch.where(keep, n, torch.zeros(()))
    with torch.inference_mode():
        r_out, n_out, _ = sm100_residual_layer_norm(
            resid.to(DEV),
            update.to(DEV),
            ln,
            final_boundary=True,
            row_valid=valid.to(DEV).view(torch.uint8),
            mask_mode=mode,
        )
    torch.testing.assert_close(r_out.cpu(), r, rtol=0, atol=1e-6)
    torch.testing.assert_close(n_out.cpu(), n, rtol=1e-5, atol=1e-5)
    if mode & 4:
        assert not n_out.cpu()[~valid].any()


# ---------------------------------------------------------------- CUDA-core attention
@pytest.mark.parametrize("head_dim", [8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize(("batch", "seq", "heads", "causal"), [(2, 128, 4, True), (1, 300, 2, False), (3, 33, 1, True)])
def test_simt_attention_head_dims(head_dim: int, batch: int, seq: int, heads: int, causal: bool) -> None:
    from solution.kernels import sm100_simt_attention

    g = torch.Generator().manual_seed(head_dim * 7 + seq)
    qkv = torch.randn(batch, seq, 3 * heads * head_dim, generator=g).to(torch.bfloat16)
    q, k, v = qkv.float().view(batch, seq, 3, heads, head_dim).permute(2, 0, 3, 1, 4).numpy()
    ref = attention_core(q, k, v, causal).transpose(0, 2, 1, 3).reshape(batch, seq, heads * head_dim)
    with torch.inference_mode():
        out, marker = sm100_simt_attention(qkv.to(DEV), heads, causal=causal)
    assert marker == "sm100_simt_attention"
    max_abs, rel = parity_errors(_bf16_np(out), ref)
    assert rel < 1e-2 and max_abs < 2e-2, (head_dim, max_abs, rel)


@pytest.mark.parametrize("head_dim", [32, 64, 256])
def test_simt_attention_key_padding_mask(head_dim: int) -> None:
    from solution.kernels import sm100_simt_attention

    batch, seq, heads = 2, 200, 2
    g = torch.Generator().manual_seed(head_dim)
    qkv = torch.randn(batch, seq, 3 * heads * head_dim, generator=g).to(torch.bfloat16)
    valid = torch.rand(batch, seq, generator=g) > 0.3
    valid[0, :40] = False  # early queries of row 0 see no valid key
    q, k, v = qkv.float().view(batch, seq, 3, heads, head_dim).permute(2, 0, 3, 1, 4).numpy()
    ref = _masked_attention_reference(q, k, v, True, valid.numpy())
    ref = ref.transpose(0, 2, 1, 3).reshape(batch, seq, heads * head_dim)
    with torch.inference_mode():
        out, _ = sm100_simt_attention(qkv.to(DEV), heads, key_valid=valid.to(DEV).view(torch.uint8))
    got = _bf16_np(out)
    assert np.isfinite(got).all() and not got[0, :40].any()
    max_abs, rel = parity_errors(got, ref)
    assert rel < 1e-2 and max_abs < 2e-2, (max_abs, rel)


# ---------------------------------------------------------------- warp-MMA attention
@pytest.mark.parametrize("head_dim", [8, 16, 32, 64, 128])
@pytest.mark.parametrize(
    ("batch", "seq", "heads", "causal"),
    [(2, 128, 4, True), (1, 300, 2, False), (3, 33, 1, True), (1, 1, 2, True), (2, 1000, 3, True), (1, 65, 1, False)],
)
def test_mma_attention_head_dims(head_dim: int, batch: int, seq: int, heads: int, causal: bool) -> None:
    from solution.kernels import sm100_mma_attention

    g = torch.Generator().manual_seed(head_dim * 11 + seq)
    qkv = torch.randn(batch, seq, 3 * heads * head_dim, generator=g).to(torch.bfloat16)
    q, k, v = qkv.float().view(batch, seq, 3, heads, head_dim).permute(2, 0, 3, 1, 4).numpy()
    ref = attention_core(q, k, v, causal).transpose(0, 2, 1, 3).reshape(batch, seq, heads * head_dim)
    with torch.inference_mode():
        out, marker = sm100_mma_attention(qkv.to(DEV), heads, causal=causal)
    assert marker == "sm100_mma_attention"
    max_abs, rel = parity_errors(_bf16_np(out), ref)
    assert rel < 1e-2 and max_abs < 2e-2, (head_dim, max_abs, rel)


@pytest.mark.parametrize("head_dim", [8, 32, 128])
def test_mma_attention_key_padding_mask_and_large_logits(head_dim: int) -> None:
    from solution.kernels import sm100_mma_attention

    batch, seq, heads = 2, 200, 2
    g = torch.Generator().manual_seed(head_dim + 5)
    qkv = torch.randn(batch, seq, 3 * heads * head_dim, generator=g)
    qkv[..., : heads * head_dim] *= 6.0  # large logits: the running max moves often
    qkv = qkv.to(torch.bfloat16)
    valid = torch.rand(batch, seq, generator=g) > 0.3
    valid[0, :40] = False  # early queries of row 0 see no valid key
    valid[1, 70:140] = False  # a whole 64-key tile of row 1 is padding
    q, k, v = qkv.float().view(batch, seq, 3, heads, head_dim).permute(2, 0, 3, 1, 4).numpy()
    ref = _masked_attention_reference(q, k, v, True, valid.numpy())
    ref = ref.transpose(0, 2, 1, 3).reshape(batch, seq, heads * head_dim)
    with torch.inference_mode():
        out, _ = sm100_mma_attention(qkv.to(DEV), heads, key_valid=valid.to(DEV).view(torch.uint8))
    got = _bf16_np(out)
    assert np.isfinite(got).all() and not got[0, :40].any()
    max_abs, rel = parity_errors(got, ref)
    assert rel < 1e-2 and max_abs < 2e-2, (max_abs, rel)


def test_mma_and_cuda_core_attention_agree_and_are_deterministic() -> None:
    from solution.kernels import sm100_mma_attention, sm100_simt_attention

    g = torch.Generator().manual_seed(32)
    qkv = torch.randn(4, 1024, 3 * 4 * 32, generator=g).to(torch.bfloat16).to(DEV)  # official_13 rows
    with torch.inference_mode():
        a, _ = sm100_mma_attention(qkv, 4)
        a2, _ = sm100_mma_attention(qkv, 4)
        b, _ = sm100_simt_attention(qkv, 4)
    assert torch.equal(a, a2)
    max_abs, rel = parity_errors(_bf16_np(a), _bf16_np(b))
    assert rel < 5e-3 and max_abs < 4e-2, (max_abs, rel)


def test_simt_and_tensor_core_attention_agree_at_head_dim_64() -> None:
    from solution.kernels import sm100_simt_attention

    g = torch.Generator().manual_seed(64)
    qkv = torch.randn(2, 700, 3 * 4 * 64, generator=g).to(torch.bfloat16).to(DEV)
    with torch.inference_mode():
        a, _ = sm100_flash_attention(qkv, 4)
        b, _ = sm100_simt_attention(qkv, 4)
    max_abs, rel = parity_errors(_bf16_np(a), _bf16_np(b))
    assert rel < 5e-3 and max_abs < 4e-2, (max_abs, rel)


# ---------------------------------------------------------------- fused block boundaries
def _bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _boundary_reference(
    resid: np.ndarray, update: np.ndarray, gamma: np.ndarray, beta: np.ndarray, update_bf16: bool,
    valid: np.ndarray | None, mask_mode: int,
) -> tuple[np.ndarray, np.ndarray]:
    u = _bf16_round(update) if update_bf16 else update.astype(np.float32)
    r = resid.astype(np.float32) + u
    if valid is not None:
        bad = ~valid
        if mask_mode & 1:
            r[bad] = resid[bad]
        if mask_mode & 2:
            r[bad] = 0.0
    n = layer_norm(r, gamma, beta)
    if valid is not None and mask_mode & 4:
        n[~valid] = 0.0
    return r, n


@pytest.mark.parametrize(
    ("rows", "width", "inner", "in_dtype", "out_dtype", "update_bf16", "mask_mode"),
    [
        (1, 32, 32, torch.float32, torch.bfloat16, True, 0),
        (63, 64, 72, torch.float32, torch.bfloat16, True, 0),  # inner % 16 != 0: zero-padded k-step
        (1000, 128, 128, torch.float32, torch.float32, False, 0),
        (129, 128, 512, torch.bfloat16, torch.bfloat16, True, 0),  # FFN-out shape, bf16 residual input
        (200, 128, 128, torch.float32, torch.bfloat16, True, 1),  # drop the update of padding rows
        (200, 32, 32, torch.float32, torch.float32, True, 2 | 4),  # zero residual and output
        # d_model 512 / 768 / 1024: the row-complete tcgen05 GEMM (CTA pair per 128-row tile)
        (1, 512, 512, torch.float32, torch.bfloat16, True, 0),  # one row of one tile
        (300, 768, 768, torch.float32, torch.bfloat16, True, 0),  # ragged last tile, 3 pieces per CTA
        (257, 512, 200, torch.float32, torch.float32, False, 0),  # last K slab partly outside x and w
        (19205, 1024, 4096, torch.bfloat16, torch.bfloat16, True, 0),  # FFN-out; pairs walk 151 tiles
        (1000, 1024, 1024, torch.float32, torch.bfloat16, True, 1),  # drop the update of padding rows
        (1000, 768, 3072, torch.float32, torch.float32, True, 2 | 4),  # zero residual and output
    ],
)
def test_linear_residual_norm(rows, width, inner, in_dtype, out_dtype, update_bf16, mask_mode) -> None:  # noqa: ANN001
    from solution.kernels import sm100_linear_residual_norm

    g = torch.Generator().manual_seed(rows + width + inner)
    x = torch.randn(rows, inner, generator=g).to(torch.bfloat16)
    w = (torch.randn(width, inner, generator=g) / inner**0.5).to(torch.bfloat16)
    b = torch.randn(width, generator=g)
    resid = (torch.randn(rows, width, generator=g) * 2).to(in_dtype)
    norm = torch.nn.LayerNorm(width)
    with torch.no_grad():
        norm.weight.normal_(generator=g)
        norm.bias.normal_(generator=g)
    valid = (torch.rand(rows, generator=g) > 0.3) if mask_mode else None
    update = x.float().numpy() @ w.float().numpy().T + b.numpy()
    r_ref, n_ref = _boundary_reference(
        resid.float().numpy(), update, norm.weight.detach().numpy(), norm.bias.detach().numpy(), update_bf16,
        None if valid is None else valid.numpy(), mask_mode,
    )
    with torch.inference_mode():
        r, n, marker = sm100_linear_residual_norm(
            x.to(DEV), w.to(DEV), b.to(DEV), resid.to(DEV), norm.to(DEV), final_boundary=out_dtype == torch.float32,
            update_dtype=torch.bfloat16 if update_bf16 else torch.float32, out_dtype=out_dtype,
            row_valid=None if valid is None else valid.to(DEV).view(torch.uint8), mask_mode=mask_mode,
        )
    assert marker == "sm100_linear_residual_norm" and n.dtype == out_dtype
    max_abs, rel = parity_errors(r.cpu().numpy(), r_ref)
    assert rel < 4e-3 and max_abs < 5e-2, ("residual", max_abs, rel)
    max_abs, rel = parity_errors(n.float().cpu().numpy(), n_ref)
    assert rel < 8e-3 and max_abs < 8e-2, ("normed", max_abs, rel)
    if valid is not None and mask_mode & 4:
        assert not n.cpu()[~valid].any()


@pytest.mark.parametrize(
    ("rows", "width", "hidden", "in_dtype", "out_dtype", "keep"),
    [
        (64, 128, 128, torch.float32, torch.bfloat16, True),  # the reference's D = F = 128
        (1000, 32, 32, torch.float32, torch.float32, False),  # official_07 widths, final boundary
        (77, 64, 256, torch.bfloat16, torch.bfloat16, True),
        (3, 128, 512, torch.float32, torch.bfloat16, True),
        (50, 64, 48, torch.float32, torch.bfloat16, True),  # the last warp's hidden slice past F
    ],
)
def test_mlp_residual_norm(rows, width, hidden, in_dtype, out_dtype, keep) -> None:  # noqa: ANN001
    from solution.kernels import sm100_mlp_residual_norm

    g = torch.Generator().manual_seed(rows * 3 + width + hidden)
    x = torch.randn(rows, width, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(hidden, width, generator=g) / width**0.5).to(torch.bfloat16)
    b1 = torch.randn(hidden, generator=g) * 0.5
    w2 = (torch.randn(width, hidden, generator=g) / hidden**0.5).to(torch.bfloat16)
    b2 = torch.randn(width, generator=g)
    resid = (torch.randn(rows, width, generator=g) * 2).to(in_dtype)
    norm = torch.nn.LayerNorm(width)
    h = _bf16_round(gelu_erf((x.float().numpy() @ w1.float().numpy().T + b1.numpy()).astype(np.float32)))
    update = h @ w2.float().numpy().T + b2.numpy()
    r_ref, n_ref = _boundary_reference(
        resid.float().numpy(), update, norm.weight.detach().numpy(), norm.bias.detach().numpy(), True, None, 0
    )
    with torch.inference_mode():
        r, n, marker = sm100_mlp_residual_norm(
            x.to(DEV), w1.to(DEV), b1.to(DEV), w2.to(DEV), b2.to(DEV), resid.to(DEV), norm.to(DEV),
            final_boundary=not keep, out_dtype=out_dtype, keep_residual=keep,
        )
    assert marker == "sm100_mlp_residual_norm" and (r is None) == (not keep)
    if keep:
        max_abs, rel = parity_errors(r.cpu().numpy(), r_ref)
        assert rel < 4e-3 and max_abs < 5e-2, ("residual", max_abs, rel)
    max_abs, rel = parity_errors(n.float().cpu().numpy(), n_ref)
    assert rel < 8e-3 and max_abs < 8e-2, ("normed", max_abs, rel)


def test_mlp_boundary_in_place_output_and_determinism() -> None:
    """The model writes the normalised output over the MLP's own input."""
    from solution.kernels import sm100_mlp_residual_norm

    g = torch.Generator().manual_seed(11)
    rows, width, hidden = 300, 128, 128
    x = torch.randn(rows, width, generator=g).to(torch.bfloat16).to(DEV)
    w1 = (torch.randn(hidden, width, generator=g) / width**0.5).to(torch.bfloat16).to(DEV)
    w2 = (torch.randn(width, hidden, generator=g) / hidden**0.5).to(torch.bfloat16).to(DEV)
    b1, b2 = torch.randn(hidden, generator=g).to(DEV), torch.randn(width, generator=g).to(DEV)
    resid = torch.randn(rows, width, generator=g).to(DEV)
    norm = torch.nn.LayerNorm(width).to(DEV)
    with torch.inference_mode():
        r1, n1, _ = sm100_mlp_residual_norm(x, w1, b1, w2, b2, resid, norm, final_boundary=False)
        r2, n2, _ = sm100_mlp_residual_norm(x, w1, b1, w2, b2, resid, norm, final_boundary=False)
        buf = x.clone()
        r3 = resid.clone()
        sm100_mlp_residual_norm(buf, w1, b1, w2, b2, r3, norm, final_boundary=False, residual_out=r3,
                                normalized_out=buf)
    assert torch.equal(n1, n2) and torch.equal(r1, r2)
    assert torch.equal(buf, n1) and torch.equal(r3, r1)
