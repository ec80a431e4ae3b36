"""b200tx_sequence_forward_noalloc: the whole forward of a small model for
callers that cannot allocate device memory.

b200tx_sequence_forward reads 192 KB of pre-swizzled weight images per layer
from memory the caller allocates.  A caller whose GPU memory is all handed out
by its framework's own pool, or that must not call cudaMalloc because it
synchronizes the device, cannot provide them; the no-alloc entry point takes
the plain bf16 weights and builds the images in a fixed 768 KB array that the
library keeps on every device (up to 4 layers).

Checked here through the C ABI, against b200tx_sequence_forward with
caller-built images (SequenceResidentForward) on the same inputs:
* two calls in a row with two different models (4 layers, then 2 layers of
  another shape), so the second call must rewrite the shared array; the same
  forward kernel reads the same image bytes, so the outputs are the same bits
  (and so well inside the parity tolerance of the other tests);
* a model with more layers than the array holds is refused with a message
  that names the limit.

The file sorts last, so that a run stopping at its first failure has run
every other test before this one.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch
from conftest import MAX_ABS_TOL, REL_L2_TOL, parity_errors

from oracle import OfficialConfig, official_input, official_state_dict
from solution import _native
from solution.runtimes.sequence_resident import SequenceResidentForward
from solution.transformer import UserOptimizedTransformer, copy_model_weights

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _clean_error_word():
    _native.device_error(clear=True)
    yield
    assert _native.device_error(clear=True) == 0, "a kernel wait timed out"


def _model(cfg: OfficialConfig, seed: int) -> UserOptimizedTransformer:
    model = UserOptimizedTransformer(SimpleNamespace(**cfg.__dict__))
    copy_model_weights(official_state_dict(cfg, seed=seed), model)
    return model.to(DEV).eval()


def _layer_weights(model: UserOptimizedTransformer):
    """The model's plain weights as b200tx_seq_layer_weights (bf16 matrices,
    fp32 vectors), the tensors that back them, ln0 and eps."""

    keep: list[torch.Tensor] = []

    def ptr(t: torch.Tensor, dtype: torch.dtype) -> int:
        v = t.detach().to(device=DEV, dtype=dtype).contiguous()
        keep.append(v)
        return v.data_ptr()

    layers = list(model.layers)
    norms = [(layer.norm1.kernel_norm(), layer.norm2.kernel_norm()) for layer in layers]
    final = model.final_norm.kernel_norm()
    rows = []
    for i, layer in enumerate(layers):
        nxt = norms[i + 1][0] if i + 1 < len(layers) else final
        rows.append(
            _native.SeqLayerWeights(
                ptr(layer.attention.qkv_proj.weight, torch.bfloat16),
                ptr(layer.attention.out_proj.weight, torch.bfloat16),
                ptr(layer.ffn_in.weight, torch.bfloat16),
                ptr(layer.ffn_out.weight, torch.bfloat16),
                ptr(layer.attention.qkv_proj.bias, torch.float32),
                ptr(layer.attention.out_proj.bias, torch.float32),
                ptr(layer.ffn_in.bias, torch.float32),
                ptr(layer.ffn_out.bias, torch.float32),
                ptr(norms[i][1].weight, torch.float32),
                ptr(norms[i][1].bias, torch.float32),
                ptr(nxt.weight, torch.float32),
                ptr(nxt.bias, torch.float32),
            )
        )
    ln0 = (ptr(norms[0][0].weight, torch.float32), ptr(norms[0][0].bias, torch.float32))
    return (_native.SeqLayerWeights * len(rows))(*rows), keep, ln0, float(final.eps)


def _noalloc_forward(model: UserOptimizedTransformer, x: torch.Tensor) -> torch.Tensor:
    layers, keep, ln0, eps = _layer_weights(model)
    out = torch.empty_like(x)
    batch, seq, d_model = x.shape
    lib = _native.load()
    rc = lib.b200tx_sequence_forward_noalloc(
        x.data_ptr(), out.data_ptr(), batch, seq, d_model, model.config.num_heads, d_model, len(layers),
        layers, ln0[0], ln0[1], eps, torch.cuda.current_stream(DEV).cuda_stream,
    )
    assert rc == 0, lib.b200tx_last_error().decode()
    torch.cuda.synchronize()
    del keep
    return out


def test_noalloc_forward_matches_the_image_entry_point_on_two_calls() -> None:
    cases = [
        (OfficialConfig(4, 128, 128, 4, 128, 4), 0, 11),  # the array's full 4 layers
        (OfficialConfig(3, 64, 128, 2, 128, 2), 1, 12),   # a second model: layers 0-1 rewritten
    ]
    for cfg, seed, x_seed in cases:
        model = _model(cfg, seed)
        x = official_input(cfg, x_seed).to(DEV)
        with torch.inference_mode():
            expected = SequenceResidentForward(model)(x)
            got = _noalloc_forward(model, x)
        torch.cuda.synchronize()
        max_abs, rel = parity_errors(got.cpu().numpy(), expected.cpu().numpy())
        assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (cfg, max_abs, rel)
        # Exact: for the second model this holds only if the call rewrote the
        # shared array with its own weights.
        assert torch.equal(got, expected), (cfg, max_abs)


def test_noalloc_forward_refuses_more_layers_than_its_array_holds() -> None:
    x = torch.zeros(1, 128, 128, device=DEV)
    out = torch.empty_like(x)
    dummy = torch.zeros(384 * 128, device=DEV)
    p = dummy.data_ptr()
    too_many = _native.SEQ_NOALLOC_MAX_LAYERS + 1
    layers = (_native.SeqLayerWeights * too_many)(*[_native.SeqLayerWeights(*([p] * 12)) for _ in range(too_many)])
    lib = _native.load()
    rc = lib.b200tx_sequence_forward_noalloc(
        x.data_ptr(), out.data_ptr(), 1, 128, 128, 4, 128, too_many, layers, p, p, 1e-5,
        torch.cuda.current_stream(DEV).cuda_stream,
    )
    assert rc == -2  # B200TX_ERR_UNSUPPORTED, before any launch
    message = lib.b200tx_last_error().decode()
    assert f"1..{_native.SEQ_NOALLOC_MAX_LAYERS}" in message and "768 KB" in message, message
