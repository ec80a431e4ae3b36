"""The libb200tx kernels as registered PyTorch operators (``torch.ops.b200tx.*``).

The reference registers its Triton kernels as functional operators with
``torch.library.triton_op("shape_aware_transformer::<name>", mutates_args={})``
(solution/shape14/triton_streaming_dh64.py:200-242,
solution/kernels/attention/triton_s1024_dh32.py:275-366) so that they trace
under meta and fake tensors (tests/solution/test_triton_shape13_attention.py:
49-79).  This module does the same for the sm100 kernels:

* ``b200tx::linear``               -- ``sm100_linear`` (bias, optional erf GELU)
* ``b200tx::flash_attention``      -- ``sm100_flash_attention`` (head_dim 64)
* ``b200tx::simt_attention``       -- ``sm100_simt_attention`` (head_dim 8..256)
* ``b200tx::mma_attention``        -- ``sm100_mma_attention`` (head_dim 8..128)
* ``b200tx::residual_layer_norm``  -- ``sm100_residual_layer_norm`` (returns
  the fp32 residual and the normalised tensor)
* ``b200tx::layer_norm``           -- ``sm100_initial_layer_norm``
* ``b200tx::linear_residual_layer_norm`` / ``b200tx::mlp_residual_layer_norm``
  -- the fused block boundaries (``sm100_linear_residual_norm`` /
  ``sm100_mlp_residual_norm``), returning ``(residual, normalised)``

Each operator is functional: it allocates its outputs and launches on the
current stream of the inputs' CUDA device.  The kernels are inference-only
(no autograd formula is registered); an operator runs them with gradient
recording off whatever the caller's grad mode is.  The fake implementations check
the same shape and dtype contract (``ValueError`` on a violation, as the
wrappers raise) and return empty outputs, so the operators trace under
``FakeTensorMode``, meta tensors and ``torch.export`` without a GPU.  A CPU
tensor raises ``RuntimeError``: there is no CPU fallback.

The model's forward calls the ctypes wrappers directly, which saves the
dispatcher's per-call cost on launch-bound shapes; these operators are the
surface for callers that trace or compose the kernels themselves.  Both
routes launch the same kernels with the same arguments, so their outputs are
bit-identical (tested on the GPU).
"""

from __future__ import annotations

import torch

from .. import _native
from .attention import (
    HEAD_DIM,
    MMA_HEAD_DIMS,
    SIMT_HEAD_DIMS,
    sm100_flash_attention,
    sm100_mma_attention,
    sm100_simt_attention,
)
from .projection import sm100_linear

NAMESPACE = "b200tx"
OPERATORS = (
    "linear",
    "flash_attention",
    "simt_attention",
    "mma_attention",
    "residual_layer_norm",
    "layer_norm",
    "linear_residual_layer_norm",
    "mlp_residual_layer_norm",
)

_IO = (torch.float32, torch.bfloat16)


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


def _no_cpu(name: str):  # noqa: ANN202 - returns a kernel for register_kernel
    def kernel(*args, **kwargs):  # noqa: ANN002, ANN003, ARG001
        raise RuntimeError(
            f"{NAMESPACE}::{name} runs only on an sm_100 CUDA device; there is no CPU fallback"
        )

    return kernel


# ---------------------------------------------------------------- linear


def _linear_shape(
    value: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, out_dtype: torch.dtype
) -> tuple[int, ...]:
    _require(value.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16,
             "value and weight must be bfloat16")
    _require(value.ndim >= 2 and weight.ndim == 2, "value must be [..., K] and weight [N, K]")
    _require(value.shape[-1] == weight.shape[1], "value and weight disagree on K")
    _require(weight.shape[1] % 8 == 0 and weight.shape[0] % 8 == 0,
             "K and N must be multiples of 8 (16-byte TMA row pitch)")
    if bias is not None:
        _require(bias.dtype == torch.float32 and tuple(bias.shape) == (weight.shape[0],),
                 "bias must be float32 [N]")
    _require(out_dtype in _IO, "out_dtype must be float32 or bfloat16")
    return (*value.shape[:-1], weight.shape[0])


@torch.library.custom_op(f"{NAMESPACE}::linear", mutates_args=(), device_types="cuda")
def linear(
    value: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    gelu: bool = False,
    out_dtype: torch.dtype = torch.bfloat16,
    variant: int = _native.GEMM_PAIR,
) -> torch.Tensor:
    """``epilogue(value . weight^T + bias)`` on the tcgen05 GEMM."""

    _linear_shape(value, weight, bias, out_dtype)
    with torch.no_grad():
        out, _ = sm100_linear(
            value.contiguous(), weight.contiguous(), bias, gelu=gelu, out_dtype=out_dtype,
            variant=variant,
        )
    return out


@linear.register_fake
def _linear_fake(value, weight, bias=None, gelu=False, out_dtype=torch.bfloat16,  # noqa: ANN001
                 variant=_native.GEMM_PAIR):  # noqa: ANN001, ANN202, ARG001
    return value.new_empty(_linear_shape(value, weight, bias, out_dtype), dtype=out_dtype)


linear.register_kernel("cpu")(_no_cpu("linear"))


# ---------------------------------------------------------------- attention


def _attention_shape(
    qkv: torch.Tensor, num_heads: int, key_valid: torch.Tensor | None, head_dims: tuple[int, ...]
) -> tuple[int, int, int]:
    _require(qkv.dtype == torch.bfloat16 and qkv.ndim == 3, "qkv must be a bfloat16 [B, S, 3D] tensor")
    _require(num_heads > 0 and qkv.shape[-1] % (3 * num_heads) == 0,
             "the packed width must be 3 * num_heads * head_dim")
    head_dim = qkv.shape[-1] // (3 * num_heads)
    _require(head_dim in head_dims, f"head_dim {head_dim} is not one of {head_dims}")
    batch, seq, width = qkv.shape
    if key_valid is not None:
        _require(key_valid.dtype == torch.uint8 and tuple(key_valid.shape) == (batch, seq),
                 "key_valid must be a uint8 [B, S] tensor")
    return batch, seq, width // 3


@torch.library.custom_op(f"{NAMESPACE}::flash_attention", mutates_args=(), device_types="cuda")
def flash_attention(
    qkv: torch.Tensor,
    num_heads: int,
    causal: bool = True,
    variant: int = _native.ATTN_QUAD,
    key_valid: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal (or full) attention over the packed projection, head_dim 64,
    on the tensor cores; returns the ``[B, S, D]`` context."""

    _attention_shape(qkv, num_heads, key_valid, (HEAD_DIM,))
    with torch.no_grad():
        out, _ = sm100_flash_attention(
            qkv.contiguous(), num_heads, causal=causal, variant=variant,
            key_valid=None if key_valid is None else key_valid.contiguous(),
        )
    return out


@flash_attention.register_fake
def _flash_attention_fake(qkv, num_heads, causal=True, variant=_native.ATTN_QUAD,  # noqa: ANN001
                          key_valid=None):  # noqa: ANN001, ANN202, ARG001
    return qkv.new_empty(_attention_shape(qkv, num_heads, key_valid, (HEAD_DIM,)))


flash_attention.register_kernel("cpu")(_no_cpu("flash_attention"))


@torch.library.custom_op(f"{NAMESPACE}::simt_attention", mutates_args=(), device_types="cuda")
def simt_attention(
    qkv: torch.Tensor,
    num_heads: int,
    causal: bool = True,
    key_valid: torch.Tensor | None = None,
) -> torch.Tensor:
    """The same attention for head_dim 8..256 on the CUDA cores."""

    _attention_shape(qkv, num_heads, key_valid, SIMT_HEAD_DIMS)
    with torch.no_grad():
        out, _ = sm100_simt_attention(
            qkv.contiguous(), num_heads, causal=causal,
            key_valid=None if key_valid is None else key_valid.contiguous(),
        )
    return out


@simt_attention.register_fake
def _simt_attention_fake(qkv, num_heads, causal=True, key_valid=None):  # noqa: ANN001, ANN202, ARG001
    return qkv.new_empty(_attention_shape(qkv, num_heads, key_valid, SIMT_HEAD_DIMS))


simt_attention.register_kernel("cpu")(_no_cpu("simt_attention"))


@torch.library.custom_op(f"{NAMESPACE}::mma_attention", mutates_args=(), device_types="cuda")
def mma_attention(
    qkv: torch.Tensor,
    num_heads: int,
    causal: bool = True,
    key_valid: torch.Tensor | None = None,
) -> torch.Tensor:
    """The same attention for head_dim 8..128 on warp-level tensor-core MMAs."""

    _attention_shape(qkv, num_heads, key_valid, MMA_HEAD_DIMS)
    with torch.no_grad():
        out, _ = sm100_mma_attention(
            qkv.contiguous(), num_heads, causal=causal,
            key_valid=None if key_valid is None else key_valid.contiguous(),
        )
    return out


@mma_attention.register_fake
def _mma_attention_fake(qkv, num_heads, causal=True, key_valid=None):  # noqa: ANN001, ANN202, ARG001
    return qkv.new_empty(_attention_shape(qkv, num_heads, key_valid, MMA_HEAD_DIMS))


mma_attention.register_kernel("cpu")(_no_cpu("mma_attention"))


# ---------------------------------------------------------------- LayerNorm


def _norm_check(
    value: torch.Tensor,
    update: torch.Tensor | None,
    weight: torch.Tensor,
    bias: torch.Tensor,
    out_dtype: torch.dtype,
    row_valid: torch.Tensor | None,
) -> None:
    _require(value.ndim >= 2 and value.dtype in _IO, "value must be a float32 or bfloat16 [..., D] tensor")
    width = value.shape[-1]
    if update is not None:
        _require(update.shape == value.shape and update.dtype in _IO,
                 "update must match value's shape, float32 or bfloat16")
    _require(
        weight.dtype == torch.float32 and bias.dtype == torch.float32
        and tuple(weight.shape) == (width,) and tuple(bias.shape) == (width,),
        "weight and bias must be float32 [D]",
    )
    _require(out_dtype in _IO, "out_dtype must be float32 or bfloat16")
    if row_valid is not None:
        _require(row_valid.dtype == torch.uint8 and row_valid.numel() == value.numel() // width,
                 "row_valid must hold one uint8 flag per row")


def _norm_launch(value, update, weight, bias, eps, out_dtype, row_valid, mask_mode, residual):  # noqa: ANN001, ANN202
    if value.device.type != "cuda" or weight.device != value.device or bias.device != value.device:
        raise RuntimeError("the sm100 LayerNorm needs value, weight and bias on one CUDA device")
    value = value.contiguous()
    normed = torch.empty(value.shape, dtype=out_dtype, device=value.device)
    _native.residual_layer_norm(
        value,
        None if update is None else update.contiguous(),
        residual,
        normed,
        weight.contiguous(),
        bias.contiguous(),
        eps,
        None if row_valid is None else row_valid.contiguous(),
        mask_mode,
    )
    return normed


@torch.library.custom_op(f"{NAMESPACE}::residual_layer_norm", mutates_args=(), device_types="cuda")
def residual_layer_norm(
    value: torch.Tensor,
    update: torch.Tensor | None,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float = 1e-5,
    out_dtype: torch.dtype = torch.bfloat16,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``r = value + update`` (fp32) and ``LN(r)``; returns ``(r, LN(r))``.
    ``row_valid`` / ``mask_mode`` apply the padding-row behaviours of the
    MASK_* bits."""

    _norm_check(value, update, weight, bias, out_dtype, row_valid)
    residual = torch.empty(value.shape, dtype=torch.float32, device=value.device)
    normed = _norm_launch(value, update, weight, bias, eps, out_dtype, row_valid, mask_mode, residual)
    return residual, normed


@residual_layer_norm.register_fake
def _residual_layer_norm_fake(value, update, weight, bias, eps=1e-5,  # noqa: ANN001
                              out_dtype=torch.bfloat16, row_valid=None,  # noqa: ANN001
                              mask_mode=0):  # noqa: ANN001, ANN202, ARG001
    _norm_check(value, update, weight, bias, out_dtype, row_valid)
    return value.new_empty(value.shape, dtype=torch.float32), value.new_empty(value.shape, dtype=out_dtype)


residual_layer_norm.register_kernel("cpu")(_no_cpu("residual_layer_norm"))


# ---------------------------------------------------------------- fused block boundaries


def _boundary_check(
    x: torch.Tensor,
    value: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    update_dtype: torch.dtype,
    out_dtype: torch.dtype,
) -> int:
    _norm_check(value, None, gamma, beta, out_dtype, None)
    width = value.shape[-1]
    _require(width in (32, 64, 128), f"the fused boundaries are built for d_model 32, 64, 128, not {width}")
    _require(x.dtype == torch.bfloat16 and x.numel() // x.shape[-1] == value.numel() // width,
             "x must be bfloat16 with one row per row of value")
    _require(update_dtype in _IO, "update_dtype must be float32 or bfloat16")
    return width


def _boundary_outputs(value: torch.Tensor, out_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    return (
        torch.empty(value.shape, dtype=torch.float32, device=value.device),
        torch.empty(value.shape, dtype=out_dtype, device=value.device),
    )


@torch.library.custom_op(f"{NAMESPACE}::linear_residual_layer_norm", mutates_args=(), device_types="cuda")
def linear_residual_layer_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    value: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float = 1e-5,
    update_dtype: torch.dtype = torch.bfloat16,
    out_dtype: torch.dtype = torch.bfloat16,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``r = value + round(x . weight^T + bias)``, ``LN(r)`` in one kernel
    (d_model 32/64/128); returns ``(r, LN(r))``."""

    width = _boundary_check(x, value, gamma, beta, update_dtype, out_dtype)
    _require(tuple(weight.shape) == (width, x.shape[-1]) and tuple(bias.shape) == (width,),
             "weight must be [D, K] and bias [D]")
    residual, normed = _boundary_outputs(value, out_dtype)
    _native.linear_residual_layer_norm(
        x.contiguous(), weight.contiguous(), bias.contiguous(), value.contiguous(), residual, normed,
        gamma.contiguous(), beta.contiguous(), eps, None, 0, update_dtype,
    )
    return residual, normed


@linear_residual_layer_norm.register_fake
def _linear_residual_layer_norm_fake(x, weight, bias, value, gamma, beta, eps=1e-5,  # noqa: ANN001
                                     update_dtype=torch.bfloat16, out_dtype=torch.bfloat16):  # noqa: ANN001, ANN202, ARG001
    width = _boundary_check(x, value, gamma, beta, update_dtype, out_dtype)
    _require(tuple(weight.shape) == (width, x.shape[-1]) and tuple(bias.shape) == (width,),
             "weight must be [D, K] and bias [D]")
    return value.new_empty(value.shape, dtype=torch.float32), value.new_empty(value.shape, dtype=out_dtype)


linear_residual_layer_norm.register_kernel("cpu")(_no_cpu("linear_residual_layer_norm"))


def _mlp_weights_check(x, w1, b1, w2, b2, width):  # noqa: ANN001, ANN202
    hidden = w1.shape[0] if w1.ndim == 2 else -1
    _require(
        hidden > 0 and hidden % 16 == 0 and x.shape[-1] == width
        and tuple(w1.shape) == (hidden, width) and tuple(w2.shape) == (width, hidden)
        and tuple(b1.shape) == (hidden,) and tuple(b2.shape) == (width,),
        "the MLP weights must be w1 [F, D], w2 [D, F], b1 [F], b2 [D] with F a multiple of 16",
    )


@torch.library.custom_op(f"{NAMESPACE}::mlp_residual_layer_norm", mutates_args=(), device_types="cuda")
def mlp_residual_layer_norm(
    x: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor,
    w2: torch.Tensor,
    b2: torch.Tensor,
    value: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float = 1e-5,
    update_dtype: torch.dtype = torch.bfloat16,
    out_dtype: torch.dtype = torch.bfloat16,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``r = value + round(bf16(GELU(x . w1^T + b1)) . w2^T + b2)``, ``LN(r)`` in
    one kernel (d_model 32/64/128); returns ``(r, LN(r))``."""

    width = _boundary_check(x, value, gamma, beta, update_dtype, out_dtype)
    _mlp_weights_check(x, w1, b1, w2, b2, width)
    residual, normed = _boundary_outputs(value, out_dtype)
    _native.mlp_residual_layer_norm(
        x.contiguous(), w1.contiguous(), b1.contiguous(), w2.contiguous(), b2.contiguous(), value.contiguous(),
        residual, normed, gamma.contiguous(), beta.contiguous(), eps, None, 0, update_dtype,
    )
    return residual, normed


@mlp_residual_layer_norm.register_fake
def _mlp_residual_layer_norm_fake(x, w1, b1, w2, b2, value, gamma, beta, eps=1e-5,  # noqa: ANN001
                                  update_dtype=torch.bfloat16, out_dtype=torch.bfloat16):  # noqa: ANN001, ANN202, ARG001
    width = _boundary_check(x, value, gamma, beta, update_dtype, out_dtype)
    _mlp_weights_check(x, w1, b1, w2, b2, width)
    return value.new_empty(value.shape, dtype=torch.float32), value.new_empty(value.shape, dtype=out_dtype)


mlp_residual_layer_norm.register_kernel("cpu")(_no_cpu("mlp_residual_layer_norm"))


@torch.library.custom_op(f"{NAMESPACE}::layer_norm", mutates_args=(), device_types="cuda")
def layer_norm(
    value: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float = 1e-5,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """``LN(value)`` with no residual add (the block's first norm1)."""

    _norm_check(value, None, weight, bias, out_dtype, None)
    return _norm_launch(value, None, weight, bias, eps, out_dtype, None, 0, None)


@layer_norm.register_fake
def _layer_norm_fake(value, weight, bias, eps=1e-5, out_dtype=torch.bfloat16):  # noqa: ANN001, ANN202, ARG001
    _norm_check(value, None, weight, bias, out_dtype, None)
    return value.new_empty(value.shape, dtype=out_dtype)


layer_norm.register_kernel("cpu")(_no_cpu("layer_norm"))


__all__ = [
    "NAMESPACE",
    "OPERATORS",
    "flash_attention",
    "layer_norm",
    "linear",
    "linear_residual_layer_norm",
    "mlp_residual_layer_norm",
    "mma_attention",
    "residual_layer_norm",
    "simt_attention",
]
