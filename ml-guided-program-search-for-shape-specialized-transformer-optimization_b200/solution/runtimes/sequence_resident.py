"""The whole forward of a small model in one launch (csrc/seq_forward_kernels.cuh).

For the reference's small official shapes (official/test_shapes.json: d_model =
ffn_dim = 128, 1-4 heads, 32-128 tokens per sequence) the per-primitive
forward of solution/transformer.py:1346-1513 is some thirty launches whose
fixed costs set the time.  ``SequenceResidentForward`` runs every layer in one
kernel instead: one CTA per 128 rows (whole sequences), the residual stream and
the accumulators in tensor memory, the weights streamed from operand images
built once here.  It follows the unfused program's rounding points (bf16
projections, probabilities and updates, fp32 residual and statistics), so its
output matches that program's within bf16 rounding.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _native

SUPPORTED_D_MODEL = 128
SUPPORTED_HEADS = (1, 2, 4)
SUPPORTED_SEQ_LENS = (32, 64, 128)
MAX_LAYERS = 8


def sequence_resident_supported(
    *, d_model: int, ffn_dim: int, num_heads: int, seq_len: int, num_layers: int, causal: bool
) -> str | None:
    """None when the whole-forward kernel is built for this model shape, else why not."""

    if d_model != SUPPORTED_D_MODEL or ffn_dim != SUPPORTED_D_MODEL:
        return f"built for d_model = ffn_dim = {SUPPORTED_D_MODEL}, not {d_model} / {ffn_dim}"
    if num_heads not in SUPPORTED_HEADS:
        return f"built for {SUPPORTED_HEADS} heads, not {num_heads}"
    if seq_len not in SUPPORTED_SEQ_LENS:
        return f"built for sequences of {SUPPORTED_SEQ_LENS} tokens, not {seq_len}"
    if not 1 <= num_layers <= MAX_LAYERS:
        return f"built for 1..{MAX_LAYERS} layers, not {num_layers}"
    if not causal:
        return "built for causal attention"
    return None


class SequenceResidentForward:
    """Weight images and per-layer pointers of one model on one device."""

    def __init__(self, model: nn.Module) -> None:
        cfg = model.config
        layers = list(model.layers)
        why = sequence_resident_supported(
            d_model=cfg.d_model, ffn_dim=cfg.ffn_dim, num_heads=cfg.num_heads, seq_len=cfg.seq_len,
            num_layers=len(layers), causal=bool(cfg.causal),
        )
        if why is not None:
            raise RuntimeError(f"the whole-forward kernel is ineligible: {why}")
        self.device = next(model.parameters()).device
        if self.device.type != "cuda":
            raise RuntimeError("the whole-forward kernel runs on CUDA devices only")
        self.heads = int(cfg.num_heads)
        d = SUPPORTED_D_MODEL
        self._keep: list[torch.Tensor] = []

        def f32(t: torch.Tensor) -> torch.Tensor:
            v = t.detach().to(device=self.device, dtype=torch.float32).contiguous()
            self._keep.append(v)
            return v

        with torch.no_grad(), torch.cuda.device(self.device):
            self.images = torch.empty((len(layers), 6, _native.SEQ_IMAGE_BYTES), dtype=torch.uint8, device=self.device)
            norms = [(layer.norm1.kernel_norm(), layer.norm2.kernel_norm()) for layer in layers]
            final = model.final_norm.kernel_norm()
            self.ln0 = (f32(norms[0][0].weight), f32(norms[0][0].bias))
            self.layers: list[_native.SeqLayer] = []
            for i, layer in enumerate(layers):
                qkv = layer.attention.qkv_proj.weight.detach().to(self.device, torch.bfloat16).contiguous()
                weights = [
                    qkv[0:d], qkv[d:2 * d], qkv[2 * d:3 * d],
                    layer.attention.out_proj.weight.detach().to(self.device, torch.bfloat16).contiguous(),
                    layer.ffn_in.weight.detach().to(self.device, torch.bfloat16).contiguous(),
                    layer.ffn_out.weight.detach().to(self.device, torch.bfloat16).contiguous(),
                ]
                for j, w in enumerate(weights):
                    _native.seq_weight_image(w.contiguous(), self.images[i, j])
                nxt = norms[i + 1][0] if i + 1 < len(layers) else final
                ptrs = [
                    f32(layer.attention.qkv_proj.bias), f32(layer.attention.out_proj.bias),
                    f32(layer.ffn_in.bias), f32(layer.ffn_out.bias),
                    f32(norms[i][1].weight), f32(norms[i][1].bias), f32(nxt.weight), f32(nxt.bias),
                ]
                self.layers.append(
                    _native.SeqLayer(self.images[i].data_ptr(), *[p.data_ptr() for p in ptrs])
                )
            self.eps = float(final.eps)
            self._layer_array = (_native.SeqLayer * len(self.layers))(*self.layers)
            torch.cuda.current_stream(self.device).synchronize()

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.device != self.device or x.dtype != torch.float32 or not x.is_contiguous() or x.dim() != 3:
            raise ValueError("x must be a contiguous float32 [B, S, 128] tensor on the model's device")
        if out is None:
            out = torch.empty_like(x)
        # Launched on the current device's stream; _native checks that it is x's device.
        _native.sequence_forward(x, out, self.heads, self._layer_array, self.ln0[0], self.ln0[1], self.eps)
        return out


__all__ = ["SequenceResidentForward", "sequence_resident_supported"]
