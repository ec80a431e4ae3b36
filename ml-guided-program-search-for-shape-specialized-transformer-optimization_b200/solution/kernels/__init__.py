"""Python wrappers over the libb200tx C ABI.

Each wrapper keeps the reference's operator conventions
(solution/shape14/triton_streaming_dh64.py:268-346,
solution/kernels/norm/triton_mixed_residual.py:80-160): ``*_available()``
reports whether the kernel library loads, ``can_use_*`` returns a bool and
never raises, and the op itself returns ``(tensor(s)..., marker)`` where the
marker names the kernel that ran.  Caller-contract violations raise
``ValueError``; ineligible inputs or a failed launch raise ``RuntimeError``.
There is no fallback path.
"""

from .attention import (
    SM100_FLASH_ATTENTION_BACKEND,
    SM100_MMA_ATTENTION_BACKEND,
    can_use_sm100_mma_attention,
    sm100_mma_attention,
    SM100_SIMT_ATTENTION_BACKEND,
    can_use_sm100_simt_attention,
    sm100_simt_attention,
    can_use_sm100_flash_attention,
    sm100_flash_attention,
    sm100_flash_attention_available,
)
from .boundary import (
    SM100_LINEAR_RESIDUAL_NORM_BACKEND,
    SM100_MLP_RESIDUAL_NORM_BACKEND,
    can_use_sm100_linear_residual_norm,
    can_use_sm100_mlp_residual_norm,
    sm100_linear_residual_norm,
    sm100_mlp_residual_norm,
)
from .norm import (
    MASK_DROP_UPDATE,
    MASK_ZERO_NORMED,
    MASK_ZERO_RESIDUAL,
    SM100_INITIAL_LAYER_NORM_BACKEND,
    SM100_RESIDUAL_LAYER_NORM_BACKEND,
    can_use_sm100_residual_layer_norm,
    sm100_initial_layer_norm,
    sm100_layer_norm_available,
    sm100_residual_layer_norm,
)
from .projection import (
    SM100_LINEAR_BACKEND,
    SM100_LINEAR_GELU_BACKEND,
    can_use_sm100_linear,
    sm100_linear,
    sm100_linear_available,
)
from . import ops  # noqa: E402 - registers the torch.ops.b200tx.* operators

__all__ = [
    "MASK_DROP_UPDATE",
    "MASK_ZERO_NORMED",
    "MASK_ZERO_RESIDUAL",
    "SM100_FLASH_ATTENTION_BACKEND",
    "SM100_MMA_ATTENTION_BACKEND",
    "can_use_sm100_mma_attention",
    "sm100_mma_attention",
    "SM100_SIMT_ATTENTION_BACKEND",
    "can_use_sm100_simt_attention",
    "sm100_simt_attention",
    "SM100_INITIAL_LAYER_NORM_BACKEND",
    "SM100_LINEAR_RESIDUAL_NORM_BACKEND",
    "SM100_MLP_RESIDUAL_NORM_BACKEND",
    "can_use_sm100_linear_residual_norm",
    "can_use_sm100_mlp_residual_norm",
    "sm100_linear_residual_norm",
    "sm100_mlp_residual_norm",
    "SM100_LINEAR_BACKEND",
    "SM100_LINEAR_GELU_BACKEND",
    "SM100_RESIDUAL_LAYER_NORM_BACKEND",
    "can_use_sm100_flash_attention",
    "can_use_sm100_linear",
    "can_use_sm100_residual_layer_norm",
    "sm100_flash_attention",
    "sm100_flash_attention_available",
    "sm100_initial_layer_norm",
    "sm100_layer_norm_available",
    "sm100_linear",
    "sm100_linear_available",
    "sm100_residual_layer_norm",
    "ops",
]
