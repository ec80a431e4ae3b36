"""Fused block boundaries for small d_model (csrc/boundary_kernels.cuh).

Replaces the reference's fused Linear residual-norm boundary
(solution/kernels/boundary/triton_linear_residual_norm.py:33-112, D 32 and
128) and its fused MLP boundary
(solution/kernels/boundary/triton_ffn_residual_norm.py:43-136, D = F = 128):
the projection that closes a branch, its bias, the rounding of the update to
the dtype the unfused program stores, the fp32 residual add and the LayerNorm
run as one kernel; the MLP form also keeps the GELU hidden row in registers.
Both are built for d_model 32, 64 and 128 (a row in one warp's registers);
the Linear form also for d_model 512, 768 and 1024, as a tcgen05 GEMM whose
CTA pair holds whole rows in tensor memory and normalises them in its
epilogue (csrc/gemm_rownorm_kernels.cuh).  Conventions as the other wrappers:
``can_use_*`` never raises, the ops return ``(residual, normalized, marker)``,
``ValueError`` for caller errors, ``RuntimeError`` for ineligible inputs.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _native
from ._common import is_sm100_cuda, launch, library_ready, require

SM100_LINEAR_RESIDUAL_NORM_BACKEND = "sm100_linear_residual_norm"
SM100_MLP_RESIDUAL_NORM_BACKEND = "sm100_mlp_residual_norm"
BOUNDARY_WIDTHS = (32, 64, 128)
LINEAR_BOUNDARY_WIDTHS = (32, 64, 128, 512, 768, 1024)
MLP_HIDDEN_MULTIPLE = 16

_IO = (torch.float32, torch.bfloat16)


def _norm_ok(layer_norm: nn.LayerNorm, width: int, device: torch.device) -> bool:
    return (
        isinstance(layer_norm, nn.LayerNorm)
        and tuple(layer_norm.normalized_shape) == (width,)
        and layer_norm.weight is not None
        and layer_norm.bias is not None
        and all(
            p.device == device and p.dtype == torch.float32 and p.is_contiguous()
            for p in (layer_norm.weight, layer_norm.bias)
        )
    )


def _bf16_matrix(t: torch.Tensor, shape: tuple[int, int], device: torch.device) -> bool:
    return (
        t.dtype == torch.bfloat16 and tuple(t.shape) == shape and t.is_contiguous()
        and t.device == device and t.data_ptr() % 16 == 0
    )


def _f32_vector(t: torch.Tensor, n: int, device: torch.device) -> bool:
    return t.dtype == torch.float32 and tuple(t.shape) == (n,) and t.is_contiguous() and t.device == device


def _common_ok(x: torch.Tensor, value: torch.Tensor, layer_norm: nn.LayerNorm, widths: tuple[int, ...]) -> bool:
    if not library_ready() or torch.is_grad_enabled() or not is_sm100_cuda(value):
        return False
    width = value.shape[-1]
    if width not in widths or value.dtype not in _IO or not value.is_contiguous():
        return False
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.device != value.device or x.data_ptr() % 16:
        return False
    if x.numel() // x.shape[-1] != value.numel() // width:
        return False
    return _norm_ok(layer_norm, width, value.device)


def can_use_sm100_linear_residual_norm(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, value: torch.Tensor, layer_norm: nn.LayerNorm
) -> bool:
    """Whether the fused Linear boundary can run on these operands (never raises)."""

    try:
        if not _common_ok(x, value, layer_norm, LINEAR_BOUNDARY_WIDTHS):
            return False
        width, inner = value.shape[-1], x.shape[-1]
        return inner % 8 == 0 and _bf16_matrix(weight, (width, inner), value.device) and _f32_vector(
            bias, width, value.device
        )
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def can_use_sm100_mlp_residual_norm(
    x: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor,
    w2: torch.Tensor,
    b2: torch.Tensor,
    value: torch.Tensor,
    layer_norm: nn.LayerNorm,
) -> bool:
    """Whether the fused MLP boundary can run on these operands (never raises)."""

    try:
        if not _common_ok(x, value, layer_norm, BOUNDARY_WIDTHS):
            return False
        width = value.shape[-1]
        if x.shape[-1] != width:
            return False
        hidden = w1.shape[0] if w1.ndim == 2 else -1
        return (
            hidden > 0 and hidden % MLP_HIDDEN_MULTIPLE == 0
            and _bf16_matrix(w1, (hidden, width), value.device)
            and _bf16_matrix(w2, (width, hidden), value.device)
            and _f32_vector(b1, hidden, value.device)
            and _f32_vector(b2, width, value.device)
        )
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def _outputs(
    value: torch.Tensor,
    *,
    final_boundary: bool,
    out_dtype: torch.dtype | None,
    residual_out: torch.Tensor | None,
    keep_residual: bool,
    normalized_out: torch.Tensor | None,
    row_valid: torch.Tensor | None,
) -> tuple[torch.Tensor | None, torch.Tensor]:
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
        require(
            residual.shape == value.shape and residual.dtype == torch.float32 and residual.is_contiguous(),
            "residual_out must be a contiguous float32 tensor of value's shape",
        )
    normalized = (
        torch.empty(value.shape, dtype=out_dtype, device=value.device) if normalized_out is None else normalized_out
    )
    require(
        normalized.shape == value.shape and normalized.dtype == out_dtype and normalized.is_contiguous(),
        f"normalized_out must be a contiguous {out_dtype} tensor of value's shape",
    )
    if row_valid is not None:
        require(
            row_valid.dtype == torch.uint8 and row_valid.device == value.device and row_valid.is_contiguous()
            and row_valid.numel() == value.numel() // value.shape[-1],
            "row_valid must be a contiguous uint8 tensor with one flag per row",
        )
    return residual, normalized


def sm100_linear_residual_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    value: torch.Tensor,
    layer_norm: nn.LayerNorm,
    *,
    final_boundary: bool,
    update_dtype: torch.dtype = torch.bfloat16,
    out_dtype: torch.dtype | None = None,
    residual_out: torch.Tensor | None = None,
    keep_residual: bool = True,
    normalized_out: torch.Tensor | None = None,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
) -> tuple[torch.Tensor | None, torch.Tensor, str]:
    """``r = value + round(x . weight^T + bias)`` and ``LN(r)`` in one kernel;
    ``update_dtype`` is the dtype the unfused program stores the update in."""

    if not can_use_sm100_linear_residual_norm(x, weight, bias, value, layer_norm):
        raise RuntimeError("sm100 fused Linear residual-norm boundary is ineligible for the requested inputs")
    require(update_dtype in _IO, "update_dtype must be float32 or bfloat16")
    residual, normalized = _outputs(
        value, final_boundary=final_boundary, out_dtype=out_dtype, residual_out=residual_out,
        keep_residual=keep_residual, normalized_out=normalized_out, row_valid=row_valid,
    )
    launch(
        _native.linear_residual_layer_norm,
        x, weight, bias, value, residual, normalized, layer_norm.weight, layer_norm.bias, layer_norm.eps,
        row_valid, mask_mode, update_dtype,
    )
    return residual, normalized, SM100_LINEAR_RESIDUAL_NORM_BACKEND


def sm100_mlp_residual_norm(
    x: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor,
    w2: torch.Tensor,
    b2: torch.Tensor,
    value: torch.Tensor,
    layer_norm: nn.LayerNorm,
    *,
    final_boundary: bool,
    update_dtype: torch.dtype = torch.bfloat16,
    out_dtype: torch.dtype | None = None,
    residual_out: torch.Tensor | None = None,
    keep_residual: bool = True,
    normalized_out: torch.Tensor | None = None,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
) -> tuple[torch.Tensor | None, torch.Tensor, str]:
    """``r = value + round(bf16(GELU(x . w1^T + b1)) . w2^T + b2)`` and ``LN(r)``
    in one kernel; the hidden activations are never written to memory."""

    if not can_use_sm100_mlp_residual_norm(x, w1, b1, w2, b2, value, layer_norm):
        raise RuntimeError("sm100 fused MLP residual-norm boundary is ineligible for the requested inputs")
    require(update_dtype in _IO, "update_dtype must be float32 or bfloat16")
    residual, normalized = _outputs(
        value, final_boundary=final_boundary, out_dtype=out_dtype, residual_out=residual_out,
        keep_residual=keep_residual, normalized_out=normalized_out, row_valid=row_valid,
    )
    launch(
        _native.mlp_residual_layer_norm,
        x, w1, b1, w2, b2, value, residual, normalized, layer_norm.weight, layer_norm.bias, layer_norm.eps,
        row_valid, mask_mode, update_dtype,
    )
    return residual, normalized, SM100_MLP_RESIDUAL_NORM_BACKEND


__all__ = [
    "BOUNDARY_WIDTHS",
    "LINEAR_BOUNDARY_WIDTHS",
    "MLP_HIDDEN_MULTIPLE",
    "SM100_LINEAR_RESIDUAL_NORM_BACKEND",
    "SM100_MLP_RESIDUAL_NORM_BACKEND",
    "can_use_sm100_linear_residual_norm",
    "can_use_sm100_mlp_residual_norm",
    "sm100_linear_residual_norm",
    "sm100_mlp_residual_norm",
]
