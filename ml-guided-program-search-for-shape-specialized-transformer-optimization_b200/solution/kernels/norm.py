"""Residual add + LayerNorm + cast on sm_100a (csrc/norm_kernels.cuh).

Replaces the reference's ``triton_initial_fp16_layer_norm``
(solution/kernels/norm/triton_initial.py:38-66), ``triton_residual_layer_norm``
(solution/kernels/norm/triton_residual.py:38-73) and
``triton_mixed_residual_layer_norm``
(solution/kernels/norm/triton_mixed_residual.py:40-160): fp32 residual stream,
bf16 normalised output, fp32 output at the final boundary.  With a padding
mask (``row_valid``, uint8 per row) the kernel also applies the reference's
``masked_fill`` of padding rows (official/torch_transformer_benchmark.py:
119-121, 143-144, 170-171; masked LayerNorm solution/kernels/norm/
triton_masked.py:47-118) per ``mask_mode``.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _native
from ._common import is_sm100_cuda, launch, library_ready, require

SM100_RESIDUAL_LAYER_NORM_BACKEND = "sm100_residual_layer_norm"
SM100_INITIAL_LAYER_NORM_BACKEND = "sm100_initial_layer_norm"

_IO = (torch.float32, torch.bfloat16)

MASK_DROP_UPDATE = _native.MASK_DROP_UPDATE
MASK_ZERO_RESIDUAL = _native.MASK_ZERO_RESIDUAL
MASK_ZERO_NORMED = _native.MASK_ZERO_NORMED


def _check_row_valid(row_valid: torch.Tensor | None, value: torch.Tensor) -> None:
    if row_valid is None:
        return
    rows = value.numel() // value.shape[-1]
    require(
        row_valid.dtype == torch.uint8
        and row_valid.device == value.device
        and row_valid.is_contiguous()
        and row_valid.numel() == rows,
        f"row_valid must be a contiguous uint8 tensor of {rows} flags on {value.device}",
    )


def sm100_layer_norm_available() -> bool:
    return library_ready()


def _norm_params_ok(layer_norm: nn.LayerNorm, width: int, device: torch.device) -> bool:
    if not isinstance(layer_norm, nn.LayerNorm):
        return False
    if tuple(layer_norm.normalized_shape) != (width,):
        return False
    if layer_norm.weight is None or layer_norm.bias is None:
        return False
    return all(
        p.device == device and p.dtype == torch.float32 and p.is_contiguous()
        for p in (layer_norm.weight, layer_norm.bias)
    )


def can_use_sm100_residual_layer_norm(
    value: torch.Tensor, update: torch.Tensor | None, layer_norm: nn.LayerNorm
) -> bool:
    """Whether the sm100 residual LayerNorm can run on these inputs (never raises)."""

    try:
        if not library_ready() or torch.is_grad_enabled() or not is_sm100_cuda(value):
            return False
        if value.ndim < 2 or not value.is_contiguous() or value.dtype not in _IO:
            return False
        if update is not None:
            if update.shape != value.shape or update.device != value.device:
                return False
            if update.dtype not in _IO or not update.is_contiguous():
                return False
        return _norm_params_ok(layer_norm, value.shape[-1], value.device)
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def sm100_residual_layer_norm(
    value: torch.Tensor,
    update: torch.Tensor,
    layer_norm: nn.LayerNorm,
    *,
    final_boundary: bool,
    out_dtype: torch.dtype | None = None,
    residual_out: torch.Tensor | None = None,
    normalized_out: torch.Tensor | None = None,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
    keep_residual: bool = True,
) -> tuple[torch.Tensor | None, torch.Tensor, str]:
    """``r = value + update`` (fp32) and ``LN(r)``.

    The normalised output is bf16 for an inner boundary and fp32 at the final
    boundary unless ``out_dtype`` says otherwise (the model passes its input
    dtype there).  ``residual_out`` may be ``value`` itself for an in-place
    update of an fp32 residual stream.  ``row_valid`` / ``mask_mode`` apply
    the padding-mask behaviours (MASK_* bits) to rows whose flag is 0.
    With ``keep_residual=False`` the sum is not written at all (the block's
    last boundary, whose residual nobody reads: 4 bytes per element less
    traffic) and the returned residual is ``None``.
    """

    if not can_use_sm100_residual_layer_norm(value, update, layer_norm):
        raise RuntimeError("sm100 residual LayerNorm is ineligible for the requested inputs")
    if out_dtype is None:
        out_dtype = torch.float32 if final_boundary else torch.bfloat16
    require(out_dtype in _IO, "out_dtype must be float32 or bfloat16")
    if not keep_residual:
        require(residual_out is None, "residual_out is given but keep_residual is False")
        residual = None
    elif residual_out is None:
        residual = torch.empty(value.shape, dtype=torch.float32, device=value.device)
    else:
        residual = residual_out
    normalized = (
        torch.empty(value.shape, dtype=out_dtype, device=value.device)
        if normalized_out is None
        else normalized_out
    )
    if residual is not None:
        require(residual.shape == value.shape and residual.dtype == torch.float32, "bad residual_out")
        require(residual.is_contiguous(), "residual_out must be contiguous")
    require(normalized.is_contiguous(), "normalized_out must be contiguous")
    require(
        normalized.shape == value.shape and normalized.dtype == out_dtype,
        f"normalized_out must be {out_dtype} of shape {tuple(value.shape)}",
    )
    _check_row_valid(row_valid, value)
    launch(
        _native.residual_layer_norm,
        value,
        update,
        residual,
        normalized,
        layer_norm.weight,
        layer_norm.bias,
        layer_norm.eps,
        row_valid,
        mask_mode,
    )
    return residual, normalized, SM100_RESIDUAL_LAYER_NORM_BACKEND


def sm100_initial_layer_norm(
    value: torch.Tensor,
    layer_norm: nn.LayerNorm,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    normalized_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, str]:
    """``LN(value)`` with no residual add (the block's first norm1)."""

    if not can_use_sm100_residual_layer_norm(value, None, layer_norm):
        raise RuntimeError("sm100 initial LayerNorm is ineligible for the requested inputs")
    require(out_dtype in _IO, "out_dtype must be float32 or bfloat16")
    normalized = (
        torch.empty(value.shape, dtype=out_dtype, device=value.device)
        if normalized_out is None
        else normalized_out
    )
    require(
        normalized.shape == value.shape and normalized.dtype == out_dtype and normalized.is_contiguous(),
        "normalized_out has the wrong shape, dtype or layout",
    )
    launch(
        _native.residual_layer_norm,
        value,
        None,
        None,
        normalized,
        layer_norm.weight,
        layer_norm.bias,
        layer_norm.eps,
    )
    return normalized, SM100_INITIAL_LAYER_NORM_BACKEND


__all__ = [
    "MASK_DROP_UPDATE",
    "MASK_ZERO_NORMED",
    "MASK_ZERO_RESIDUAL",
    "SM100_INITIAL_LAYER_NORM_BACKEND",
    "SM100_RESIDUAL_LAYER_NORM_BACKEND",
    "can_use_sm100_residual_layer_norm",
    "sm100_initial_layer_norm",
    "sm100_layer_norm_available",
    "sm100_residual_layer_norm",
]
