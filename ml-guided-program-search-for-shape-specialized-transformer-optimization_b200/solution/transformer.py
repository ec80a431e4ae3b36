"""Official-compatible Transformer whose forward runs on the sm_100a kernels.

Public contract of the reference's ``solution/transformer.py``:
``UserOptimizedTransformer(config)`` (:1065-1109) with the official
constructor, ``forward(x, valid_token_mask=None)`` (:1677-1791),
``configure_execution(*, config)`` (:1227-1236), ``describe_execution_path()``
(:1323-1337), ``set_execution_observation()`` (:1339-1344) and
``copy_model_weights`` (:1806-1871, q/k/v packed into one ``qkv_proj``).

The block is the official pre-LN causal block
(official/torch_transformer_benchmark.py:125-172):
    x = x + out_proj(attention(LN1(x)))
    x = x + ffn_out(GELU_erf(ffn_in(LN2(x))))
    y = final_norm(x)
executed as one packed-QKV GEMM, one flash-attention launch, one out-proj
GEMM, one fused residual+LayerNorm, one GEMM with a bias+GELU epilogue, one
GEMM and one fused residual+LayerNorm per layer (plus the initial LayerNorm):
seven launches per layer, every one a libb200tx kernel.  The residual stream
is fp32; GEMM operands and attention inputs are bf16 with fp32 accumulation;
the output has the input's dtype.
"""

from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from typing import Any

import torch
from torch import nn

from .config import (
    AttentionBackend,
    ConfigSpec,
    FFNBackend,
    ResidualNormBackend,
    RuntimeBackend,
    portable_config,
)
from .kernels import (
    MASK_DROP_UPDATE,
    MASK_ZERO_NORMED,
    MASK_ZERO_RESIDUAL,
    SM100_FLASH_ATTENTION_BACKEND,
    SM100_MMA_ATTENTION_BACKEND,
    SM100_SIMT_ATTENTION_BACKEND,
    SM100_INITIAL_LAYER_NORM_BACKEND,
    SM100_LINEAR_BACKEND,
    SM100_LINEAR_GELU_BACKEND,
    SM100_RESIDUAL_LAYER_NORM_BACKEND,
    sm100_flash_attention,
    sm100_mma_attention,
    sm100_simt_attention,
    sm100_initial_layer_norm,
    sm100_linear,
    sm100_residual_layer_norm,
)
from .kernels.boundary import (
    SM100_LINEAR_RESIDUAL_NORM_BACKEND,
    SM100_MLP_RESIDUAL_NORM_BACKEND,
    sm100_linear_residual_norm,
    sm100_mlp_residual_norm,
)
from .plan import ExecutionContext, ExecutionPlan
from .plan_builder import PlanBuilder
from .runtimes import BatchTiledGraphReplay, CudaGraphReplay

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def _strict_backend_marker(actual: str, *, expected_marker: str, planned_backend: str) -> str:
    """Normalise a primitive's marker or expose an implementation drift.

    Reference: solution/transformer.py:275-288.
    """

    if actual != expected_marker:
        raise RuntimeError(
            "execution backend marker does not match the compiled plan: "
            f"expected marker {expected_marker!r}, received {actual!r}"
        )
    return planned_backend


@dataclass(slots=True)
class _ExecutionObservation:
    """What actually ran, in the vocabulary of ``ExpectedExecutionTrace``.

    Reference: solution/transformer.py:102-238.
    """

    config_id: str
    runtime_backend: str = RuntimeBackend.EAGER.value
    calls: dict[str, int] = field(default_factory=dict)
    backends: dict[str, set[str]] = field(default_factory=dict)
    dtypes: dict[str, set[str]] = field(default_factory=dict)

    def record(self, role: str, backend: str, dtype: torch.dtype | None = None) -> None:
        self.calls[role] = self.calls.get(role, 0) + 1
        self.backends.setdefault(role, set()).add(backend)
        if dtype is not None:
            self.dtypes.setdefault(role, set()).add(str(dtype).removeprefix("torch."))

    def to_signature(self, plan: ExecutionPlan) -> dict[str, Any]:
        """Observed signature; equal to the expected one when the plan ran as built."""

        expected = plan.expected_trace.to_dict()
        observed = dict(expected)

        def single(role: str) -> str | None:
            values = self.backends.get(role, set())
            return next(iter(values)) if len(values) == 1 else None

        def single_dtype(role: str) -> str | None:
            values = self.dtypes.get(role, set())
            return next(iter(values)) if len(values) == 1 else None

        observed["runtime_backend"] = self.runtime_backend
        for role, key in (
            ("attention", "attention_backend"),
            ("qkv_projection", "qkv_projection_backend"),
            ("attention_output_projection", "attention_output_projection_backend"),
            ("ffn_input_projection", "ffn_input_projection_backend"),
            ("ffn_output_projection", "ffn_output_projection_backend"),
            ("residual_norm", "residual_norm_backend"),
            ("initial_norm", "initial_norm_backend"),
            ("ffn", "ffn_backend"),
        ):
            observed[key] = single(role)
            observed[f"{role}_calls"] = self.calls.get(role, 0)
        for role, key in (
            ("attention", "attention_compute_dtype"),
            ("qkv_projection", "qkv_projection_compute_dtype"),
            ("attention_output_projection", "attention_output_projection_compute_dtype"),
            ("ffn_input_projection", "ffn_input_projection_compute_dtype"),
            ("ffn_output_projection", "ffn_output_projection_compute_dtype"),
            ("ffn_activation", "ffn_activation_output_dtype"),
        ):
            observed[key] = single_dtype(role)
        observed["runtime_calls"] = 1
        observed["config_id"] = self.config_id
        return observed


class KernelEventRecorder:
    """Optional per-primitive CUDA-event timing of the eager forward.

    When installed on a model (``model.kernel_events = KernelEventRecorder()``)
    every primitive launch is bracketed by two CUDA events on the stream it is
    launched on; ``durations_ms()`` sums them per role after a synchronise.
    Inside a CUDA-graph capture nothing is recorded.
    """

    def __init__(self) -> None:
        self.events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def start(self, role: str) -> Any:
        if torch.cuda.is_current_stream_capturing():
            return None
        begin = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        begin.record()
        return (role, begin, end)

    def stop(self, token: Any) -> None:
        if token is None:
            return
        token[2].record()
        self.events.append(token)

    def durations_ms(self) -> dict[str, list[float]]:
        torch.cuda.synchronize()
        out: dict[str, list[float]] = {}
        for role, begin, end in self.events:
            out.setdefault(role, []).append(begin.elapsed_time(end))
        return out

    def clear(self) -> None:
        self.events.clear()


class _NoRecorder:
    @staticmethod
    def start(role: str) -> None:
        return None

    @staticmethod
    def stop(token: Any) -> None:
        return None


_NO_RECORDER = _NoRecorder()


class _Bf16ShadowLinear(nn.Linear):
    """Linear layer with non-persistent bf16 inference weights.

    Reference: ``_FP16ShadowLinear`` (solution/transformer.py:291-353); the
    fp32 parameters stay the source of truth, the shadow is derived once per
    device move or weight load.  The bias stays fp32 (the GEMM epilogue adds it
    in fp32).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True) -> None:
        super().__init__(in_features, out_features, bias=bias)
        self.register_buffer("_bf16_shadow_weight", None, persistent=False)
        self.register_buffer("_f32_shadow_bias", None, persistent=False)

    def materialize_bf16_shadow(self) -> None:
        if self._bf16_shadow_weight is not None:
            return
        self._bf16_shadow_weight = self.weight.detach().to(torch.bfloat16).contiguous()
        self._f32_shadow_bias = (
            None if self.bias is None else self.bias.detach().to(torch.float32).contiguous()
        )

    def clear_bf16_shadow(self) -> None:
        self._bf16_shadow_weight = None
        self._f32_shadow_bias = None

    def shadow_parameters(self) -> tuple[torch.Tensor, torch.Tensor | None]:
        if self._bf16_shadow_weight is None:
            raise RuntimeError("bf16 shadow weights must be materialised before use")
        return self._bf16_shadow_weight, self._f32_shadow_bias


class _Fp32LayerNorm(nn.LayerNorm):
    """LayerNorm whose affine parameters are handed to the kernels in fp32."""

    def kernel_norm(self) -> nn.LayerNorm:
        if self.weight.dtype == torch.float32 and self.bias.dtype == torch.float32:
            return self
        shadow = getattr(self, "_f32_shadow", None)
        if shadow is None:
            shadow = nn.LayerNorm(self.normalized_shape, eps=self.eps, device=self.weight.device)
            with torch.no_grad():
                shadow.weight.copy_(self.weight.float())
                shadow.bias.copy_(self.bias.float())
            shadow.requires_grad_(False)
            object.__setattr__(self, "_f32_shadow", shadow)
        return shadow

    def clear_shadow(self) -> None:
        object.__setattr__(self, "_f32_shadow", None)


class _SelfAttention(nn.Module):
    """Packed QKV projection and output projection of one block."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.qkv_proj = _Bf16ShadowLinear(d_model, 3 * d_model, bias=True)
        self.out_proj = _Bf16ShadowLinear(d_model, d_model, bias=True)


class _TransformerBlock(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = _Fp32LayerNorm(d_model)
        self.attention = _SelfAttention(d_model, num_heads)
        self.norm2 = _Fp32LayerNorm(d_model)
        self.ffn_in = _Bf16ShadowLinear(d_model, ffn_dim)
        self.ffn_out = _Bf16ShadowLinear(ffn_dim, d_model)


class UserOptimizedTransformer(nn.Module):
    """Solution entry with the official constructor and forward API."""

    def __init__(self, config: Any) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [
                _TransformerBlock(config.d_model, config.num_heads, config.ffn_dim)
                for _ in range(config.num_layers)
            ]
        )
        self.final_norm = _Fp32LayerNorm(config.d_model)

        self._cuda_graph_replay: CudaGraphReplay | None = None
        self._batch_tiled_graph_replay: BatchTiledGraphReplay | None = None
        self._sequence_resident: Any = None  # SequenceResidentForward, built on first use
        self._shadows_ready = False
        self._runtime_plan_signature: tuple[object, ...] | None = None
        self._runtime_plan: ExecutionPlan | None = None
        self._execution_observation_enabled = False
        self._last_execution_observation: dict[str, Any] | None = None
        self._classified_mask: torch.Tensor | None = None
        self._classified_mask_version: int | None = None
        self._classified_mask_is_all_valid = False
        self._plan_builder = PlanBuilder()
        self._explicit_config: ConfigSpec | None = None
        self._active_config = portable_config(head_dim=int(config.d_model) // int(config.num_heads))
        # Where the active config came from: "deployed" (an exact entry of
        # deployment/deployed_configs.json for this environment and shape),
        # "default" (no entry matched) or "explicit" (configure_execution).
        self.active_config_source = "default"
        self._deployment_signature: tuple[object, ...] | None = None
        self.kernel_events: KernelEventRecorder | None = None
        self.register_load_state_dict_post_hook(_after_weight_load)

    # ------------------------------------------------------------ state
    def _invalidate_runtime_state(self) -> None:
        self._cuda_graph_replay = None
        self._batch_tiled_graph_replay = None
        self._sequence_resident = None
        self._runtime_plan_signature = None
        self._runtime_plan = None
        self._last_execution_observation = None
        self._classified_mask = None
        self._classified_mask_version = None
        self._classified_mask_is_all_valid = False

    def _apply(self, function: Any, recurse: bool = True) -> UserOptimizedTransformer:
        result = super()._apply(function, recurse=recurse)
        self._clear_shadow_weights()
        self._invalidate_runtime_state()
        self._deployment_signature = None
        if self._explicit_config is None and next(self.parameters()).is_cuda:
            self._resolve_default_config()
        return result

    def _materialize_shadow_weights(self) -> None:
        # A no-op once done; a weight load, a device move or a clear resets it.
        if self._shadows_ready:
            return
        for module in self.modules():
            if isinstance(module, _Bf16ShadowLinear):
                module.materialize_bf16_shadow()
        self._shadows_ready = True

    def _clear_shadow_weights(self) -> None:
        self._shadows_ready = False
        for module in self.modules():
            if isinstance(module, _Bf16ShadowLinear):
                module.clear_bf16_shadow()
            elif isinstance(module, _Fp32LayerNorm):
                module.clear_shadow()
        # Captured graphs hold pointers to the old shadows; the whole-forward
        # runtime holds copies of the old weights.
        self._cuda_graph_replay = None
        self._batch_tiled_graph_replay = None
        self._sequence_resident = None

    # ------------------------------------------------------------ config
    def _resolve_default_config(self, value: torch.Tensor | None = None) -> None:
        """Resolve one exact deployed config, else the default sm100 program.

        Reference: solution/transformer.py:1144-1225.
        """

        if self._explicit_config is not None:
            return
        parameter = next(self.parameters())
        device = parameter.device if value is None else value.device
        dtype = parameter.dtype if value is None else value.dtype
        shape = (
            (self.config.batch_size, self.config.seq_len, self.config.d_model)
            if value is None
            else tuple(value.shape)
        )
        # Training and autograd state are part of the key: a deployed config
        # rejected while the module was still in training mode (at .to(),
        # before .eval()) is resolved again for the inference forward.
        grad = torch.is_grad_enabled() if value is not None else False
        signature = (device.type, device.index, dtype, shape, self.training, grad)
        if signature == self._deployment_signature:
            return
        from .shape14.defaults import default_streamed_config, is_streamed_shape

        resolved: ConfigSpec | None = None
        if device.type == "cuda":
            from deployment.environment import ImplementationScope
            from deployment.registry import (
                EnvironmentFingerprint,
                ShapeFingerprint,
                resolve_deployed_config,
            )

            scope = (
                ImplementationScope.SHAPE14
                if is_streamed_shape(shape[1], shape[2])
                else ImplementationScope.RESIDENT
            )
            try:
                hardware = EnvironmentFingerprint.detect(device, scope=scope)
                resolved = resolve_deployed_config(
                    hardware=hardware,
                    shape=ShapeFingerprint(
                        batch_size=int(shape[0]),
                        qkv_dim=int(self.config.d_model),
                        heads=int(self.config.num_heads),
                        seq_len=int(shape[1]),
                        layers=int(self.config.num_layers),
                        causal=bool(self.config.causal),
                        ffn_dim=int(self.config.ffn_dim),
                        dtype=str(dtype).removeprefix("torch."),
                        padding_ratio=0.0,
                        input_scale=1.0,
                    ),
                )
            except (FileNotFoundError, ValueError, RuntimeError):
                resolved = None
        if resolved is not None and not self._plan_builder.evaluate(
            resolved, self._execution_context(value)
        ).accepted:
            resolved = None
        selected = resolved or (
            default_streamed_config(int(shape[0]))
            if is_streamed_shape(shape[1], shape[2])
            else portable_config(head_dim=int(self.config.d_model) // int(self.config.num_heads))
        )
        if selected != self._active_config:
            self._invalidate_runtime_state()
        self._active_config = selected
        self.active_config_source = "deployed" if resolved is not None else "default"
        self._deployment_signature = signature

    @property
    def active_config(self) -> ConfigSpec:
        return self._active_config

    def configure_execution(self, *, config: ConfigSpec) -> None:
        """Install one explicit config after strict compilation for this model."""

        if not isinstance(config, ConfigSpec):
            raise TypeError("config must be ConfigSpec")
        self._plan_builder.build(config, self._execution_context())
        self._invalidate_runtime_state()
        self._explicit_config = config
        self._active_config = config
        self.active_config_source = "explicit"
        self._deployment_signature = None

    def _execution_context(
        self,
        value: torch.Tensor | None = None,
        valid_token_mask: torch.Tensor | None = None,
    ) -> ExecutionContext:
        parameter = next(self.parameters())
        if value is None:
            device = parameter.device
            dtype = parameter.dtype
            shape = (self.config.batch_size, self.config.seq_len, self.config.d_model)
            contiguous, has_mask, mask_ok, grad = True, False, True, False
        else:
            device = value.device
            dtype = value.dtype
            shape = tuple(value.shape)
            contiguous = value.is_contiguous()
            has_mask = valid_token_mask is not None
            mask_ok = valid_token_mask is None or (
                valid_token_mask.device == value.device
                and valid_token_mask.dtype == torch.bool
                and valid_token_mask.ndim == 2
                and tuple(valid_token_mask.shape) == tuple(value.shape[:2])
            )
            grad = torch.is_grad_enabled()
        return ExecutionContext(
            batch_size=shape[0],
            seq_len=shape[1],
            d_model=shape[-1],
            num_heads=self.config.num_heads,
            causal=bool(self.config.causal),
            device=device,
            dtype=dtype,
            training=self.training,
            grad_enabled=grad,
            input_contiguous=contiguous,
            has_valid_token_mask=has_mask,
            mask_compatible=mask_ok,
            ffn_dim=self.config.ffn_dim,
            num_layers=self.config.num_layers,
        )

    def _execution_plan(
        self, value: torch.Tensor | None = None, valid_token_mask: torch.Tensor | None = None
    ) -> ExecutionPlan:
        return self._plan_builder.build(
            self._active_config, self._execution_context(value, valid_token_mask)
        )

    def _cached_execution_plan(
        self, value: torch.Tensor, valid_token_mask: torch.Tensor | None
    ) -> ExecutionPlan:
        mask_sig = None
        if valid_token_mask is not None:
            mask_sig = (valid_token_mask.device, valid_token_mask.dtype, tuple(valid_token_mask.shape))
        signature = (
            self._active_config.config_id,
            value.device,
            value.dtype,
            tuple(value.shape),
            value.is_contiguous(),
            mask_sig,
            self.training,
            torch.is_grad_enabled(),
        )
        if signature != self._runtime_plan_signature:
            self._runtime_plan = self._execution_plan(value, valid_token_mask)
            self._runtime_plan_signature = signature
        assert self._runtime_plan is not None
        return self._runtime_plan

    def describe_execution_path(self) -> dict[str, Any]:
        """Describe the last plan, or a preview before the first execution."""

        plan = self._runtime_plan or self._execution_plan()
        description = plan.describe()
        expected = plan.expected_trace.to_dict()
        expected["config_id"] = plan.config_id
        description.update(
            requested_config_id=self._active_config.config_id,
            planned_config_id=plan.config_id,
            runtime_backend=plan.runtime_backend.value,
            expected_execution_signature=expected,
            observed_execution_signature=self._last_execution_observation,
        )
        return description

    def set_execution_observation(self, enabled: bool) -> None:
        self._execution_observation_enabled = bool(enabled)
        if enabled:
            self._cuda_graph_replay = None
            self._batch_tiled_graph_replay = None
            self._last_execution_observation = None

    def _effective_valid_token_mask(
        self, value: torch.Tensor, valid_token_mask: torch.Tensor | None
    ) -> torch.Tensor | None:
        """Collapse an unchanged all-valid mask once per tensor (one host sync).

        Reference: solution/transformer.py:1646-1675.
        """

        if valid_token_mask is None:
            return None
        if not (
            valid_token_mask.device == value.device
            and valid_token_mask.dtype == torch.bool
            and valid_token_mask.ndim == 2
            and tuple(valid_token_mask.shape) == tuple(value.shape[:2])
        ):
            return valid_token_mask
        try:
            version = valid_token_mask._version
        except RuntimeError:
            return None if bool(valid_token_mask.all().item()) else valid_token_mask
        if self._classified_mask is not valid_token_mask or self._classified_mask_version != version:
            self._classified_mask = valid_token_mask
            self._classified_mask_version = version
            self._classified_mask_is_all_valid = bool(valid_token_mask.all().item())
        return None if self._classified_mask_is_all_valid else valid_token_mask

    # ------------------------------------------------------------ execution
    def _forward_eager(
        self,
        value: torch.Tensor,
        valid_token_mask: torch.Tensor | None,
        plan: ExecutionPlan,
        *,
        observe: bool = True,
        out: torch.Tensor | None = None,
        defer_final: bool = False,
    ) -> Any:
        """One pass of the planned program over ``value`` ([B, S, D], contiguous).

        Returns the output ([B, S, D] in the input's dtype; ``out`` when given).
        With ``defer_final`` the output is not written yet: the return value
        is ``finish(out)``, which launches the pass's last kernel (the final
        residual LayerNorm, or the fused boundary that ends the last block)
        into ``out``.  The graph runtimes capture everything before it and
        call ``finish`` after each replay with a freshly allocated output, so
        no captured buffer is ever copied out.
        """

        observation = (
            _ExecutionObservation(config_id=plan.config_id)
            if observe and self._execution_observation_enabled
            else None
        )
        batch, seq, d_model = value.shape
        rows = batch * seq
        device = value.device
        heads = self.config.num_heads
        causal = bool(self.config.causal)
        out_update = _DTYPES[plan.attention_output_update_dtype]
        ffn_update = _DTYPES[plan.ffn_output_update_dtype]
        n_layers = len(self.layers)
        attention_variant = (
            plan.attention_launch.kernel_variant if plan.attention_launch is not None else 0
        )
        simt_attention = plan.attention_backend is AttentionBackend.SM100_SIMT
        mma_attention = plan.attention_backend is AttentionBackend.SM100_MMA
        attention_marker = (
            SM100_SIMT_ATTENTION_BACKEND
            if simt_attention
            else SM100_MMA_ATTENTION_BACKEND
            if mma_attention
            else SM100_FLASH_ATTENTION_BACKEND
        )

        # Fused block boundaries (small d_model): the out-projection and the
        # FFN-out run inside the residual-LayerNorm kernel, and with the fused
        # MLP so do the FFN-in and GELU (reference: solution/transformer.py:844,
        # 1410-1440).
        fused_boundary = plan.residual_norm_backend is ResidualNormBackend.SM100_LINEAR_MIXED
        fused_mlp = plan.ffn_backend is FFNBackend.SM100_FUSED_MLP_BOUNDARY

        def gemm_variant(launch: Any) -> int:
            return launch.kernel_variant if launch is not None else 1  # the CTA-pair GEMM

        qkv_variant = gemm_variant(plan.qkv_launch)
        out_proj_variant = gemm_variant(plan.attention_output_projection_launch)
        ffn_in_variant = gemm_variant(plan.ffn_input_launch)
        ffn_out_variant = gemm_variant(plan.ffn_launch)

        flat_in = value.reshape(rows, d_model)

        def finish(close: Any) -> Any:
            """Run (or hand back) the closing launch of the pass."""

            def into(target: torch.Tensor) -> torch.Tensor:
                close(target.view(rows, d_model))
                return target

            if defer_final:
                return into
            return into(
                out if out is not None else torch.empty((batch, seq, d_model), dtype=value.dtype, device=device)
            )

        # Padding mask (official/torch_transformer_benchmark.py:105-121,
        # 143-144, 170-171): keys of padding tokens are masked in attention,
        # their attention output is dropped, each block's output rows and the
        # final output rows are zeroed.  The bool mask is read as uint8 flags
        # in place (no copy for a contiguous mask).
        key_valid = None
        row_valid = None
        if valid_token_mask is not None:
            key_valid = valid_token_mask.contiguous().view(torch.uint8)
            row_valid = key_valid.view(rows)
        if n_layers == 0:

            def close_norm_only(normalized_out: torch.Tensor) -> None:
                if row_valid is None:
                    sm100_initial_layer_norm(
                        flat_in, self.final_norm.kernel_norm(), out_dtype=value.dtype, normalized_out=normalized_out
                    )
                else:
                    sm100_residual_layer_norm(
                        flat_in,
                        None,
                        self.final_norm.kernel_norm(),
                        final_boundary=True,
                        out_dtype=value.dtype,
                        normalized_out=normalized_out,
                        row_valid=row_valid,
                        mask_mode=MASK_ZERO_NORMED,
                    )

            return finish(close_norm_only)

        residual = torch.empty((rows, d_model), dtype=torch.float32, device=device)
        normalized = torch.empty((rows, d_model), dtype=torch.bfloat16, device=device)
        qkv = torch.empty((batch, seq, 3 * d_model), dtype=torch.bfloat16, device=device)
        context = torch.empty((batch, seq, d_model), dtype=torch.bfloat16, device=device)
        attn_update = (
            None if fused_boundary else torch.empty((rows, d_model), dtype=out_update, device=device)
        )
        hidden = (
            None if fused_mlp else torch.empty((rows, self.config.ffn_dim), dtype=torch.bfloat16, device=device)
        )
        ffn_out = (
            None
            if fused_boundary
            else attn_update
            if ffn_update == out_update
            else torch.empty((rows, d_model), dtype=ffn_update, device=device)
        )

        rec = self.kernel_events or _NO_RECORDER

        def ffn_half(index: int, layer: _TransformerBlock, last: bool) -> Any:
            """The FFN of block ``index`` up to its closing launch, which is
            returned as ``close(normalized_out)``: the residual LayerNorm (or
            the fused boundary) that adds the FFN update to the residual and
            normalises with the next block's norm1, or the final norm after
            the last block."""

            w_1, b_1 = layer.ffn_in.shadow_parameters()
            w_2, b_2 = layer.ffn_out.shadow_parameters()
            next_norm = self.final_norm if last else self.layers[index + 1].norm1
            boundary = dict(
                final_boundary=last,
                update_dtype=ffn_update,
                out_dtype=value.dtype if last else torch.bfloat16,
                residual_out=None if last else residual,
                keep_residual=not last,
                row_valid=row_valid,
                mask_mode=MASK_ZERO_RESIDUAL | (MASK_ZERO_NORMED if last else 0),
            )
            if fused_mlp:

                def close(normalized_out: torch.Tensor) -> None:
                    # Each CTA stages its rows of `normalized` before it writes
                    # them back normalised, so the in-place output is safe.
                    token = rec.start("residual_norm")
                    _, _, marker = sm100_mlp_residual_norm(
                        normalized, w_1, b_1, w_2, b_2, residual, next_norm.kernel_norm(),
                        normalized_out=normalized_out, **boundary,
                    )
                    rec.stop(token)
                    _strict_backend_marker(
                        marker,
                        expected_marker=SM100_MLP_RESIDUAL_NORM_BACKEND,
                        planned_backend=plan.ffn_backend.value,
                    )

                return close
            token = rec.start("ffn_input_projection")
            _, marker = sm100_linear(normalized, w_1, b_1, gelu=True, out=hidden, variant=ffn_in_variant)
            rec.stop(token)
            _strict_backend_marker(
                marker,
                expected_marker=SM100_LINEAR_GELU_BACKEND,
                planned_backend=plan.ffn_input_projection_backend.value,
            )
            if fused_boundary:

                def close(normalized_out: torch.Tensor) -> None:
                    token = rec.start("residual_norm")
                    _, _, marker = sm100_linear_residual_norm(
                        hidden, w_2, b_2, residual, next_norm.kernel_norm(),
                        normalized_out=normalized_out, **boundary,
                    )
                    rec.stop(token)
                    _strict_backend_marker(
                        marker,
                        expected_marker=SM100_LINEAR_RESIDUAL_NORM_BACKEND,
                        planned_backend=plan.residual_norm_backend.value,
                    )

                return close
            token = rec.start("ffn_output_projection")
            _, marker = sm100_linear(hidden, w_2, b_2, out_dtype=ffn_update, out=ffn_out, variant=ffn_out_variant)
            rec.stop(token)
            _strict_backend_marker(
                marker,
                expected_marker=SM100_LINEAR_BACKEND,
                planned_backend=plan.ffn_output_projection_backend.value,
            )
            norm_args = {k: v for k, v in boundary.items() if k != "update_dtype"}

            def close(normalized_out: torch.Tensor) -> None:
                token = rec.start("residual_norm")
                _, _, marker = sm100_residual_layer_norm(
                    residual, ffn_out, next_norm.kernel_norm(), normalized_out=normalized_out, **norm_args
                )
                rec.stop(token)
                _strict_backend_marker(
                    marker,
                    expected_marker=SM100_RESIDUAL_LAYER_NORM_BACKEND,
                    planned_backend=plan.residual_norm_backend.value,
                )

            return close

        token = rec.start("initial_norm")
        _, marker = sm100_initial_layer_norm(
            flat_in, self.layers[0].norm1.kernel_norm(), normalized_out=normalized
        )
        rec.stop(token)
        _strict_backend_marker(
            marker,
            expected_marker=SM100_INITIAL_LAYER_NORM_BACKEND,
            planned_backend=plan.initial_norm_backend.value,
        )
        if observation is not None:
            observation.record("initial_norm", plan.initial_norm_backend.value)

        residual_source = flat_in
        qkv_flat = qkv.view(rows, 3 * d_model)
        context_flat = context.view(rows, d_model)
        for index, layer in enumerate(self.layers):
            attention = layer.attention
            w_qkv, b_qkv = attention.qkv_proj.shadow_parameters()
            token = rec.start("qkv_projection")
            _, marker = sm100_linear(normalized, w_qkv, b_qkv, out=qkv_flat, variant=qkv_variant)
            rec.stop(token)
            _strict_backend_marker(
                marker,
                expected_marker=SM100_LINEAR_BACKEND,
                planned_backend=plan.qkv_projection_backend.value,
            )
            token = rec.start("attention")
            if simt_attention:
                _, marker = sm100_simt_attention(qkv, heads, causal=causal, out=context, key_valid=key_valid)
            elif mma_attention:
                _, marker = sm100_mma_attention(qkv, heads, causal=causal, out=context, key_valid=key_valid)
            else:
                _, marker = sm100_flash_attention(
                    qkv, heads, causal=causal, out=context, variant=attention_variant, key_valid=key_valid
                )
            rec.stop(token)
            _strict_backend_marker(
                marker,
                expected_marker=attention_marker,
                planned_backend=plan.attention_backend.value,
            )
            w_o, b_o = attention.out_proj.shadow_parameters()
            if fused_boundary:
                token = rec.start("residual_norm")
                _, _, marker = sm100_linear_residual_norm(
                    context_flat,
                    w_o,
                    b_o,
                    residual_source,
                    layer.norm2.kernel_norm(),
                    final_boundary=False,
                    update_dtype=out_update,
                    residual_out=residual,
                    normalized_out=normalized,
                    row_valid=row_valid,
                    mask_mode=MASK_DROP_UPDATE,
                )
                rec.stop(token)
                _strict_backend_marker(
                    marker,
                    expected_marker=SM100_LINEAR_RESIDUAL_NORM_BACKEND,
                    planned_backend=plan.residual_norm_backend.value,
                )
            else:
                token = rec.start("attention_output_projection")
                _, marker = sm100_linear(
                    context_flat, w_o, b_o, out_dtype=out_update, out=attn_update, variant=out_proj_variant
                )
                rec.stop(token)
                _strict_backend_marker(
                    marker,
                    expected_marker=SM100_LINEAR_BACKEND,
                    planned_backend=plan.attention_output_projection_backend.value,
                )
                token = rec.start("residual_norm")
                _, _, marker = sm100_residual_layer_norm(
                    residual_source,
                    attn_update,
                    layer.norm2.kernel_norm(),
                    final_boundary=False,
                    residual_out=residual,
                    normalized_out=normalized,
                    row_valid=row_valid,
                    mask_mode=MASK_DROP_UPDATE,
                )
                rec.stop(token)
                _strict_backend_marker(
                    marker,
                    expected_marker=SM100_RESIDUAL_LAYER_NORM_BACKEND,
                    planned_backend=plan.residual_norm_backend.value,
                )
            residual_source = residual
            last = index == n_layers - 1
            close_block = ffn_half(index, layer, last)
            if not last:
                close_block(normalized)
            if observation is not None:
                observation.record("qkv_projection", plan.qkv_projection_backend.value, qkv.dtype)
                observation.record("attention", plan.attention_backend.value, qkv.dtype)
                observation.record(
                    "attention_output_projection",
                    plan.attention_output_projection_backend.value,
                    context.dtype,
                )
                observation.record("residual_norm", plan.residual_norm_backend.value)
                observation.record("ffn", plan.ffn_backend.value)
                observation.record(
                    "ffn_input_projection", plan.ffn_input_projection_backend.value, normalized.dtype
                )
                observation.record("ffn_activation", "gelu", torch.bfloat16)
                observation.record(
                    "ffn_output_projection", plan.ffn_output_projection_backend.value, torch.bfloat16
                )
                observation.record("residual_norm", plan.residual_norm_backend.value)
        if observation is not None:
            self._last_execution_observation = observation.to_signature(plan)
        return finish(close_block)

    def forward(
        self, x: torch.Tensor, valid_token_mask: torch.Tensor | None = None
    ) -> torch.Tensor:
        if x.is_cuda and x.device.index != torch.cuda.current_device():
            # The kernel library works on the current device: make it the
            # input's for this call (a model on cuda:1 called while cuda:0 is
            # current).
            with torch.cuda.device(x.device):
                return self.forward(x, valid_token_mask)
        self._resolve_default_config(x)
        valid_token_mask = self._effective_valid_token_mask(x, valid_token_mask)
        plan = self._cached_execution_plan(x, valid_token_mask)
        self._materialize_shadow_weights()

        def program(
            value: torch.Tensor,
            mask: torch.Tensor | None,
            *,
            out: torch.Tensor | None = None,
            defer_final: bool = False,
        ) -> Any:
            return self._forward_eager(value, mask, plan, out=out, defer_final=defer_final)

        with torch.inference_mode():
            if plan.use_sequence_resident:
                # The whole forward in one kernel; its weight images are built
                # on first use (and again after any weight load or device move).
                from .runtimes.sequence_resident import SequenceResidentForward

                if self._sequence_resident is None or self._sequence_resident.device != x.device:
                    self._sequence_resident = SequenceResidentForward(self)
                output = self._sequence_resident(x)
                if self._execution_observation_enabled:
                    self._last_execution_observation = {
                        "runtime_backend": RuntimeBackend.SEQUENCE_RESIDENT.value,
                        "kernel": "sm100_sequence_forward",
                        "runtime_calls": 1,
                    }
                return output
            if plan.use_streamed_execution:
                from .shape14.executor import execute_streamed

                microbatch = plan.microbatch_size
                if microbatch is None or microbatch <= 0:
                    raise RuntimeError("streamed plan is missing its microbatch size")
                output = execute_streamed(
                    x, valid_token_mask, microbatch_size=microbatch, forward_chunk=program
                )
                self._mark_runtime(RuntimeBackend.STREAMED)
                return output
            if plan.use_batch_tiled_cuda_graph:
                if plan.batch_tile_size is None:
                    raise RuntimeError("batch-tiled plan is missing its tile size")
                if self._batch_tiled_graph_replay is None:
                    self._batch_tiled_graph_replay = BatchTiledGraphReplay(plan.batch_tile_size)
                output = self._batch_tiled_graph_replay.run(program, x, valid_token_mask)
                self._mark_runtime(RuntimeBackend.BATCH_TILED_CUDA_GRAPH)
                return output
            if plan.use_cuda_graph:
                if self._cuda_graph_replay is None:
                    self._cuda_graph_replay = CudaGraphReplay(
                        reuse_unchanged_input=plan.reuse_unchanged_input
                    )
                output = self._cuda_graph_replay.run(program, x, valid_token_mask)
                self._mark_runtime(RuntimeBackend.CUDA_GRAPH)
                return output
            return program(x, valid_token_mask)

    def _mark_runtime(self, runtime: RuntimeBackend) -> None:
        if self._execution_observation_enabled and self._last_execution_observation is not None:
            self._last_execution_observation["runtime_backend"] = runtime.value


def _after_weight_load(module: nn.Module, incompatible_keys: Any) -> None:
    """Any load_state_dict invalidates the derived bf16/fp32 shadows."""

    if isinstance(module, UserOptimizedTransformer):
        module._clear_shadow_weights()
        module._invalidate_runtime_state()


def _packed_source_keys(target_key: str) -> tuple[str, str, str] | None:
    marker = ".attention.qkv_proj."
    if marker not in target_key:
        return None
    prefix, suffix = target_key.split(marker, maxsplit=1)
    base = f"{prefix}.attention."
    return tuple(f"{base}{name}.{suffix}" for name in ("q_proj", "k_proj", "v_proj"))  # type: ignore[return-value]


def copy_model_weights(
    baseline: nn.Module | dict[str, torch.Tensor],
    optimized: nn.Module,
    strict: bool = True,
) -> None:
    """Copy official weights and pack q/k/v into each ``qkv_proj`` once.

    ``baseline`` is the official module (or its state dict).  Reference:
    solution/transformer.py:1806-1871.
    """

    source = baseline if isinstance(baseline, dict) else baseline.state_dict()
    target = optimized.state_dict()
    mapped: dict[str, torch.Tensor] = {}
    consumed: set[str] = set()
    for key, tensor in target.items():
        packed = _packed_source_keys(key)
        if packed is None:
            if key in source:
                mapped[key] = source[key]
                consumed.add(key)
            continue
        if not all(name in source for name in packed):
            continue
        stacked = torch.cat([source[name] for name in packed], dim=0)
        if stacked.shape != tensor.shape:
            raise RuntimeError(
                f"packed tensor shape mismatch for {key}: source={tuple(stacked.shape)}, "
                f"target={tuple(tensor.shape)}"
            )
        mapped[key] = stacked
        consumed.update(packed)
    missing = sorted(set(target) - set(mapped))
    unused = sorted(set(source) - consumed)
    if strict and (missing or unused):
        raise RuntimeError(
            f"strict weight mapping failed; missing target keys={missing}, unused source keys={unused}"
        )
    incompatible = optimized.load_state_dict(mapped, strict=strict)
    clear = getattr(optimized, "_clear_shadow_weights", None)
    if callable(clear):
        clear()
    if not strict:
        parts = []
        if missing or incompatible.missing_keys:
            parts.append(f"missing target keys={sorted(set(missing + incompatible.missing_keys))}")
        if unused:
            parts.append(f"unused source keys={unused}")
        if incompatible.unexpected_keys:
            parts.append(f"unexpected mapped keys={sorted(incompatible.unexpected_keys)}")
        if parts:
            warnings.warn("non-strict weight mapping: " + ", ".join(parts), RuntimeWarning, stacklevel=2)


__all__ = ["KernelEventRecorder", "UserOptimizedTransformer", "copy_model_weights"]
