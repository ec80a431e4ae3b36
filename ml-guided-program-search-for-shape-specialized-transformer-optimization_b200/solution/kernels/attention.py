"""Causal flash attention on the sm_100a tensor cores (csrc/attention_kernels.cuh).

Replaces the reference's streaming Dh64 kernel
(solution/shape14/triton_streaming_dh64.py:68-346), the shape13 kernel
(solution/kernels/attention/triton_s1024_dh32.py:72-366), the SDPA and
query-blocked reference operators (solution/operators/attention/sdpa.py:76-170)
and ``split_qkv`` (solution/operators/projection/qkv_layout.py:22-50): the
kernel reads Q/K/V head tiles straight out of the packed ``[B, S, 3D]`` QKV
projection and writes the ``[B, S, D]`` context the out-projection consumes.
A ``key_valid`` padding mask (uint8 ``[B, S]``) masks padding keys with -inf
as the official block does (official/torch_transformer_benchmark.py:105-108).
"""

from __future__ import annotations

import torch

from .. import _native
from ._common import is_sm100_cuda, launch, library_ready, require

SM100_FLASH_ATTENTION_BACKEND = "sm100_flash_attention"
HEAD_DIM = 64


def sm100_flash_attention_available() -> bool:
    return library_ready()


def can_use_sm100_flash_attention(qkv: torch.Tensor, num_heads: int) -> bool:
    """Whether the flash kernel can read this packed projection (never raises)."""

    try:
        if not library_ready() or torch.is_grad_enabled() or not is_sm100_cuda(qkv):
            return False
        if qkv.dtype != torch.bfloat16 or qkv.ndim != 3 or not qkv.is_contiguous():
            return False
        if num_heads <= 0 or qkv.shape[-1] != 3 * num_heads * HEAD_DIM:
            return False
        return qkv.data_ptr() % 16 == 0
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def sm100_flash_attention(
    qkv: torch.Tensor,
    num_heads: int,
    *,
    causal: bool = True,
    out: torch.Tensor | None = None,
    variant: int = _native.ATTN_QUAD,
    key_valid: torch.Tensor | None = None,
) -> tuple[torch.Tensor, str]:
    """``softmax(q k^T / 8 [+ causal] [+ key padding]) v`` per head; returns
    the ``[B, S, D]`` context.  With ``key_valid`` the QUAD, DUO and
    PERSISTENT variants are built; a query that sees no valid key gets a zero
    row."""

    if not can_use_sm100_flash_attention(qkv, num_heads):
        raise RuntimeError("sm100 flash attention is ineligible for the requested inputs")
    batch, seq, width = qkv.shape
    d_model = width // 3
    result = (
        torch.empty((batch, seq, d_model), dtype=torch.bfloat16, device=qkv.device)
        if out is None
        else out
    )
    require(
        tuple(result.shape) == (batch, seq, d_model)
        and result.dtype == torch.bfloat16
        and result.is_contiguous()
        and result.data_ptr() % 16 == 0,
        "out must be a contiguous, 16-byte aligned bf16 [B, S, D] tensor",
    )
    if key_valid is not None:
        require(
            key_valid.dtype == torch.uint8
            and key_valid.device == qkv.device
            and key_valid.is_contiguous()
            and tuple(key_valid.shape) == (batch, seq),
            "key_valid must be a contiguous uint8 [B, S] tensor on the qkv device",
        )
        require(
            variant in (_native.ATTN_QUAD, _native.ATTN_PERSISTENT, _native.ATTN_DUO, _native.ATTN_PINGPONG),
            "padding masks are built into the QUAD, PERSISTENT, DUO and PINGPONG variants only",
        )
    launch(
        _native.attention,
        qkv,
        result,
        batch,
        seq,
        num_heads,
        HEAD_DIM,
        HEAD_DIM**-0.5,
        causal,
        variant,
        key_valid,
    )
    return result, SM100_FLASH_ATTENTION_BACKEND


SM100_SIMT_ATTENTION_BACKEND = "sm100_simt_attention"
SIMT_HEAD_DIMS = (8, 16, 32, 64, 128, 256)


def can_use_sm100_simt_attention(qkv: torch.Tensor, num_heads: int) -> bool:
    """Whether the CUDA-core attention can read this packed projection (never raises)."""

    try:
        if not library_ready() or torch.is_grad_enabled() or not is_sm100_cuda(qkv):
            return False
        if qkv.dtype != torch.bfloat16 or qkv.ndim != 3 or not qkv.is_contiguous():
            return False
        if num_heads <= 0 or qkv.shape[-1] % (3 * num_heads):
            return False
        return qkv.shape[-1] // (3 * num_heads) in SIMT_HEAD_DIMS and qkv.data_ptr() % 16 == 0
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def sm100_simt_attention(
    qkv: torch.Tensor,
    num_heads: int,
    *,
    causal: bool = True,
    out: torch.Tensor | None = None,
    key_valid: torch.Tensor | None = None,
) -> tuple[torch.Tensor, str]:
    """The same attention as ``sm100_flash_attention`` for head_dim 8..256 on
    the CUDA cores (csrc/attention_simt_kernels.cuh); the official benchmark
    shapes of the reference need head dims 8, 32, 128 and 256."""

    if not can_use_sm100_simt_attention(qkv, num_heads):
        raise RuntimeError("sm100 CUDA-core attention is ineligible for the requested inputs")
    batch, seq, width = qkv.shape
    d_model = width // 3
    head_dim = d_model // num_heads
    result = (
        torch.empty((batch, seq, d_model), dtype=torch.bfloat16, device=qkv.device)
        if out is None
        else out
    )
    require(
        tuple(result.shape) == (batch, seq, d_model)
        and result.dtype == torch.bfloat16
        and result.is_contiguous()
        and result.data_ptr() % 16 == 0,
        "out must be a contiguous, 16-byte aligned bf16 [B, S, D] tensor",
    )
    if key_valid is not None:
        require(
            key_valid.dtype == torch.uint8
            and key_valid.device == qkv.device
            and key_valid.is_contiguous()
            and tuple(key_valid.shape) == (batch, seq),
            "key_valid must be a contiguous uint8 [B, S] tensor on the qkv device",
        )
    launch(
        _native.attention_generic,
        qkv,
        result,
        batch,
        seq,
        num_heads,
        head_dim,
        head_dim**-0.5,
        causal,
        key_valid,
    )
    return result, SM100_SIMT_ATTENTION_BACKEND


SM100_MMA_ATTENTION_BACKEND = "sm100_mma_attention"
MMA_HEAD_DIMS = (8, 16, 32, 64, 128)


def can_use_sm100_mma_attention(qkv: torch.Tensor, num_heads: int) -> bool:
    """Whether the warp-MMA attention can read this packed projection (never raises)."""

    try:
        if not library_ready() or torch.is_grad_enabled() or not is_sm100_cuda(qkv):
            return False
        if qkv.dtype != torch.bfloat16 or qkv.ndim != 3 or not qkv.is_contiguous():
            return False
        if num_heads <= 0 or qkv.shape[-1] % (3 * num_heads):
            return False
        return qkv.shape[-1] // (3 * num_heads) in MMA_HEAD_DIMS and qkv.data_ptr() % 16 == 0
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def sm100_mma_attention(
    qkv: torch.Tensor,
    num_heads: int,
    *,
    causal: bool = True,
    out: torch.Tensor | None = None,
    key_valid: torch.Tensor | None = None,
) -> tuple[torch.Tensor, str]:
    """The same attention as ``sm100_flash_attention`` for head_dim 8, 16, 32, 64
    and 128 on warp-level tensor-core MMAs (csrc/attention_mma_kernels.cuh),
    for the short sequences of the reference's official shapes."""

    if not can_use_sm100_mma_attention(qkv, num_heads):
        raise RuntimeError("sm100 warp-MMA attention is ineligible for the requested inputs")
    batch, seq, width = qkv.shape
    d_model = width // 3
    head_dim = d_model // num_heads
    result = (
        torch.empty((batch, seq, d_model), dtype=torch.bfloat16, device=qkv.device)
        if out is None
        else out
    )
    require(
        tuple(result.shape) == (batch, seq, d_model)
        and result.dtype == torch.bfloat16
        and result.is_contiguous()
        and result.data_ptr() % 16 == 0,
        "out must be a contiguous, 16-byte aligned bf16 [B, S, D] tensor",
    )
    if key_valid is not None:
        require(
            key_valid.dtype == torch.uint8
            and key_valid.device == qkv.device
            and key_valid.is_contiguous()
            and tuple(key_valid.shape) == (batch, seq),
            "key_valid must be a contiguous uint8 [B, S] tensor on the qkv device",
        )
    launch(
        _native.attention_mma,
        qkv,
        result,
        batch,
        seq,
        num_heads,
        head_dim,
        head_dim**-0.5,
        causal,
        key_valid,
    )
    return result, SM100_MMA_ATTENTION_BACKEND


__all__ = [
    "HEAD_DIM",
    "MMA_HEAD_DIMS",
    "SM100_MMA_ATTENTION_BACKEND",
    "can_use_sm100_mma_attention",
    "sm100_mma_attention",
    "SIMT_HEAD_DIMS",
    "SM100_SIMT_ATTENTION_BACKEND",
    "can_use_sm100_simt_attention",
    "sm100_simt_attention",
    "SM100_FLASH_ATTENTION_BACKEND",
    "can_use_sm100_flash_attention",
    "sm100_flash_attention",
    "sm100_flash_attention_available",
]
