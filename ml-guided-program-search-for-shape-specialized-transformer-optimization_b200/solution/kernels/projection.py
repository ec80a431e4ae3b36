"""Linear projections on the sm_100a tensor cores (csrc/gemm_kernels.cuh).

Replaces the reference's ``triton_qkv_native_bhsd``
(solution/kernels/projection/triton_qkv_layout.py:59-113),
``triton_attention_output_projection``
(solution/kernels/projection/triton_attention_output.py:69-147),
``triton_linear_exact_gelu`` (solution/kernels/ffn/triton_linear_exact_gelu.py:68-132)
and the fp16-shadow ``F.linear`` (solution/transformer.py:333-353):
``out = epilogue(value . weight^T + bias)`` with bf16 operands and fp32
accumulation; the epilogue adds the fp32 bias and optionally applies the exact
erf GELU before the cast.
"""

from __future__ import annotations

import torch

from .. import _native
from ._common import is_sm100_cuda, launch, library_ready, require

SM100_LINEAR_BACKEND = "sm100_linear"
SM100_LINEAR_GELU_BACKEND = "sm100_linear_gelu"

_OUT = (torch.float32, torch.bfloat16)


def sm100_linear_available() -> bool:
    return library_ready()


def can_use_sm100_linear(
    value: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None
) -> bool:
    """Whether the tcgen05 GEMM can run on these operands (never raises)."""

    try:
        if not library_ready() or torch.is_grad_enabled() or not is_sm100_cuda(value):
            return False
        if value.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
            return False
        if value.ndim < 2 or weight.ndim != 2 or value.shape[-1] != weight.shape[1]:
            return False
        if not value.is_contiguous() or not weight.is_contiguous():
            return False
        if weight.device != value.device:
            return False
        k, n = weight.shape[1], weight.shape[0]
        if k % 8 or n % 8:
            return False
        if value.data_ptr() % 16 or weight.data_ptr() % 16:
            return False
        if bias is not None:
            if bias.dtype != torch.float32 or bias.shape != (n,) or not bias.is_contiguous():
                return False
            if bias.device != value.device:
                return False
        return True
    except Exception:  # noqa: BLE001 - predicate contract: never raise
        return False


def sm100_linear(
    value: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    gelu: bool = False,
    out_dtype: torch.dtype = torch.bfloat16,
    out: torch.Tensor | None = None,
    variant: int = _native.GEMM_PAIR,
) -> tuple[torch.Tensor, str]:
    """``[..., K] x [N, K]^T -> [..., N]`` on the tensor cores; ``variant``
    picks the built kernel (``GEMM_1SM`` 128x256 tiles per SM, ``GEMM_PAIR``
    256x256 tiles per CTA pair)."""

    if not can_use_sm100_linear(value, weight, bias):
        raise RuntimeError("sm100 linear is ineligible for the requested operands")
    require(out_dtype in _OUT, "out_dtype must be float32 or bfloat16")
    shape = (*value.shape[:-1], weight.shape[0])
    result = torch.empty(shape, dtype=out_dtype, device=value.device) if out is None else out
    require(
        tuple(result.shape) == shape and result.dtype == out_dtype and result.is_contiguous(),
        "out has the wrong shape, dtype or layout",
    )
    require(result.data_ptr() % 16 == 0, "out must be 16-byte aligned")
    launch(
        _native.linear,
        value,
        weight,
        bias,
        result,
        _native.EPI_BIAS_GELU if gelu else _native.EPI_BIAS,
        variant,
    )
    return result, SM100_LINEAR_GELU_BACKEND if gelu else SM100_LINEAR_BACKEND


__all__ = [
    "SM100_LINEAR_BACKEND",
    "SM100_LINEAR_GELU_BACKEND",
    "can_use_sm100_linear",
    "sm100_linear",
    "sm100_linear_available",
]
