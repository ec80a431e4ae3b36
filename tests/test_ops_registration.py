"""The registered operators ``torch.ops.b200tx.*`` (solution/kernels/ops.py).

Mirrors the reference's fake-implementation test
(tests/solution/test_triton_shape13_attention.py:49-79): every operator traces
on meta tensors, under ``FakeTensorMode`` and through ``torch.export`` with no
GPU, and reports the output shapes and dtypes the kernels produce.  Contract
violations raise ``ValueError`` at trace time; a CPU tensor raises
``RuntimeError`` (no CPU fallback).  The GPU tests check that each operator
gives the same bits as the direct wrapper and pass ``torch.library.opcheck``.
"""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from solution import _native
from solution.kernels import (
    ops,
    sm100_flash_attention,
    sm100_linear,
    sm100_mma_attention,
    sm100_residual_layer_norm,
    sm100_simt_attention,
)

B200 = torch.ops.b200tx


def _meta(*shape, dtype=torch.bfloat16):  # noqa: ANN001, ANN002, ANN202
    return torch.empty(*shape, device="meta", dtype=dtype)


def test_every_operator_is_registered_with_a_schema() -> None:
    for name in ops.OPERATORS:
        schema = str(getattr(B200, name).default._schema)
        assert schema.startswith(f"b200tx::{name}(")
    assert "Tensor? bias=None" in str(B200.linear.default._schema)
    assert str(B200.residual_layer_norm.default._schema).endswith("-> (Tensor, Tensor)")


def test_operators_trace_on_meta_tensors() -> None:
    y = B200.linear(_meta(2, 128, 256), _meta(1024, 256), _meta(1024, dtype=torch.float32), True)
    assert (y.device.type, tuple(y.shape), y.dtype) == ("meta", (2, 128, 1024), torch.bfloat16)
    y = B200.linear(_meta(300, 64), _meta(16, 64), None, out_dtype=torch.float32)
    assert (tuple(y.shape), y.dtype) == ((300, 16), torch.float32)

    ctx = B200.flash_attention(_meta(4, 333, 3 * 1024), 16)
    assert (tuple(ctx.shape), ctx.dtype) == ((4, 333, 1024), torch.bfloat16)
    ctx = B200.flash_attention(_meta(2, 10, 3 * 128), 2, False, _native.ATTN_DUO,
                               _meta(2, 10, dtype=torch.uint8))
    assert tuple(ctx.shape) == (2, 10, 128)
    ctx = B200.simt_attention(_meta(3, 17, 3 * 32), 4)  # head_dim 8
    assert tuple(ctx.shape) == (3, 17, 32)
    ctx = B200.mma_attention(_meta(3, 17, 3 * 128), 4)  # head_dim 32
    assert tuple(ctx.shape) == (3, 17, 128)

    gamma, beta = _meta(768, dtype=torch.float32), _meta(768, dtype=torch.float32)
    r, n = B200.residual_layer_norm(_meta(5, 7, 768, dtype=torch.float32), _meta(5, 7, 768),
                                    gamma, beta, 1e-5, torch.float32)
    assert (tuple(r.shape), r.dtype, n.dtype) == ((5, 7, 768), torch.float32, torch.float32)
    n = B200.layer_norm(_meta(9, 768, dtype=torch.float32), gamma, beta)
    assert (tuple(n.shape), n.dtype) == ((9, 768), torch.bfloat16)

    g128, b128 = _meta(128, dtype=torch.float32), _meta(128, dtype=torch.float32)
    r, n = B200.linear_residual_layer_norm(_meta(40, 512), _meta(128, 512), g128,
                                           _meta(40, 128, dtype=torch.float32), g128, b128)
    assert (tuple(r.shape), r.dtype, n.dtype) == ((40, 128), torch.float32, torch.bfloat16)
    r, n = B200.mlp_residual_layer_norm(_meta(2, 20, 128), _meta(256, 128), _meta(256, dtype=torch.float32),
                                        _meta(128, 256), g128, _meta(2, 20, 128, dtype=torch.float32),
                                        g128, b128, out_dtype=torch.float32)
    assert (tuple(n.shape), n.dtype) == ((2, 20, 128), torch.float32)


def test_operators_trace_under_fake_tensor_mode() -> None:
    with FakeTensorMode():
        x = torch.empty(8, 64, 3 * 256, dtype=torch.bfloat16)
        ctx = B200.flash_attention(x, 4)
        w = torch.empty(512, 256, dtype=torch.bfloat16)
        y = B200.linear(ctx, w, torch.empty(512), gelu=True)
        assert tuple(y.shape) == (8, 64, 512)
        r, n = B200.residual_layer_norm(torch.empty(8, 64, 512), y, torch.empty(512), torch.empty(512))
        assert (r.dtype, n.dtype) == (torch.float32, torch.bfloat16)


class _Block(torch.nn.Module):
    """Attention + out-projection + residual LayerNorm, through the operators."""

    def __init__(self) -> None:
        super().__init__()
        self.w_o = torch.nn.Parameter(torch.zeros(128, 128, dtype=torch.bfloat16), requires_grad=False)
        self.b_o = torch.nn.Parameter(torch.zeros(128), requires_grad=False)
        self.gamma = torch.nn.Parameter(torch.ones(128), requires_grad=False)
        self.beta = torch.nn.Parameter(torch.zeros(128), requires_grad=False)

    def forward(self, residual: torch.Tensor, qkv: torch.Tensor) -> torch.Tensor:
        ctx = torch.ops.b200tx.flash_attention(qkv, 2)
        u = torch.ops.b200tx.linear(ctx, self.w_o, self.b_o)
        _, normed = torch.ops.b200tx.residual_layer_norm(residual, u, self.gamma, self.beta)
        return normed


def test_operators_export_as_graph_nodes() -> None:
    residual = torch.zeros(2, 16, 128)
    qkv = torch.zeros(2, 16, 3 * 128, dtype=torch.bfloat16)
    exported = torch.export.export(_Block(), (residual, qkv))
    targets = [str(node.target) for node in exported.graph.nodes if node.op == "call_function"]
    assert "b200tx.flash_attention.default" in targets
    assert "b200tx.linear.default" in targets
    assert "b200tx.residual_layer_norm.default" in targets


@pytest.mark.parametrize(
    ("call", "message"),
    [
        (lambda: B200.linear(_meta(4, 64), _meta(16, 32), None), "disagree on K"),
        (lambda: B200.linear(_meta(4, 60), _meta(16, 60), None), "multiples of 8"),
        (lambda: B200.linear(_meta(4, 64, dtype=torch.float32), _meta(16, 64), None), "bfloat16"),
        (lambda: B200.linear(_meta(4, 64), _meta(16, 64), _meta(8, dtype=torch.float32)), "bias"),
        (lambda: B200.flash_attention(_meta(2, 8, 3 * 96), 2), "head_dim 48"),
        (lambda: B200.flash_attention(_meta(2, 8, 3 * 128), 2, True, _native.ATTN_QUAD,
                                      _meta(2, 9, dtype=torch.uint8)), "key_valid"),
        (lambda: B200.simt_attention(_meta(2, 8, 3 * 96), 1), "head_dim 96"),
        (lambda: B200.mma_attention(_meta(2, 8, 3 * 512), 2), "head_dim 256"),
        (lambda: B200.linear_residual_layer_norm(_meta(4, 256), _meta(256, 256), _meta(256, dtype=torch.float32),
                                                 _meta(4, 256, dtype=torch.float32), _meta(256, dtype=torch.float32),
                                                 _meta(256, dtype=torch.float32)), "d_model 32, 64, 128"),
        (lambda: B200.mlp_residual_layer_norm(_meta(4, 64), _meta(40, 64), _meta(40, dtype=torch.float32),
                                              _meta(64, 40), _meta(64, dtype=torch.float32),
                                              _meta(4, 64, dtype=torch.float32), _meta(64, dtype=torch.float32),
                                              _meta(64, dtype=torch.float32)), "multiple of 16"),
        (lambda: B200.layer_norm(_meta(4, 64, dtype=torch.float32), _meta(32, dtype=torch.float32),
                                 _meta(32, dtype=torch.float32)), "weight and bias"),
        (lambda: B200.residual_layer_norm(_meta(4, 64, dtype=torch.float32), _meta(4, 32),
                                          _meta(64, dtype=torch.float32),
                                          _meta(64, dtype=torch.float32)), "update"),
    ],
)
def test_contract_violations_raise_value_error_at_trace_time(call, message: str) -> None:  # noqa: ANN001
    with pytest.raises(ValueError, match=message):
        call()


def test_cpu_tensors_raise_runtime_error() -> None:
    a = torch.zeros(4, 64, dtype=torch.bfloat16)
    w = torch.zeros(16, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        B200.linear(a, w, None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        B200.flash_attention(torch.zeros(1, 4, 3 * 64, dtype=torch.bfloat16), 1)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        B200.layer_norm(torch.zeros(4, 64), torch.ones(64), torch.zeros(64))


# ---------------------------------------------------------------- GPU

DEV = torch.device("cuda", 0)


@pytest.fixture
def _clean_error_word():  # noqa: ANN202
    _native.device_error(clear=True)
    yield
    assert _native.device_error(clear=True) == 0, "a kernel wait timed out"


@pytest.mark.gpu
@pytest.mark.usefixtures("_clean_error_word")
def test_operators_match_the_wrappers_bit_for_bit() -> None:
    g = torch.Generator(device=DEV).manual_seed(7)
    qkv = torch.randn(2, 300, 3 * 256, device=DEV, generator=g).to(torch.bfloat16)
    with torch.inference_mode():
        for variant in (_native.ATTN_QUAD, _native.ATTN_DUO, _native.ATTN_PERSISTENT):
            want, _ = sm100_flash_attention(qkv, 4, variant=variant)
            got = B200.flash_attention(qkv, 4, True, variant)
            assert torch.equal(got, want)
        want, _ = sm100_mma_attention(qkv, 8)  # head_dim 32
        assert torch.equal(B200.mma_attention(qkv, 8), want)
        want, _ = sm100_simt_attention(qkv, 8)
        assert torch.equal(B200.simt_attention(qkv, 8), want)

        ctx = want
        w = (torch.randn(512, 256, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
        bias = torch.randn(512, device=DEV, generator=g)
        for gelu in (False, True):
            want, _ = sm100_linear(ctx, w, bias, gelu=gelu)
            assert torch.equal(B200.linear(ctx, w, bias, gelu), want)

        ln = torch.nn.LayerNorm(512).to(DEV)
        ln.weight.normal_(generator=g)
        residual = torch.randn(2, 300, 512, device=DEV, generator=g)
        update, _ = sm100_linear(ctx, w, bias)
        r_want, n_want, _ = sm100_residual_layer_norm(residual, update, ln, final_boundary=False)
        r_got, n_got = B200.residual_layer_norm(residual, update, ln.weight, ln.bias, ln.eps)
        assert torch.equal(r_got, r_want) and torch.equal(n_got, n_want)


@pytest.mark.gpu
@pytest.mark.usefixtures("_clean_error_word")
def test_opcheck_on_the_gpu() -> None:
    g = torch.Generator(device=DEV).manual_seed(3)
    qkv = torch.randn(1, 130, 3 * 128, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(128, 128, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn(128, device=DEV, generator=g)
    gamma, beta = torch.ones(128, device=DEV), torch.zeros(128, device=DEV)
    ctx = B200.flash_attention(qkv, 2)
    utils = ("test_schema", "test_faketensor")
    torch.library.opcheck(B200.flash_attention.default, (qkv, 2), test_utils=utils)
    torch.library.opcheck(B200.simt_attention.default, (qkv, 4), test_utils=utils)
    torch.library.opcheck(B200.mma_attention.default, (qkv, 4), test_utils=utils)
    torch.library.opcheck(B200.linear.default, (ctx, w, bias, True), test_utils=utils)
    torch.library.opcheck(B200.residual_layer_norm.default,
                          (torch.randn(1, 130, 128, device=DEV), ctx, gamma, beta), test_utils=utils)
    torch.library.opcheck(B200.layer_norm.default, (ctx, gamma, beta), test_utils=utils)
    residual = torch.randn(1, 130, 128, device=DEV, generator=g)
    torch.library.opcheck(B200.linear_residual_layer_norm.default, (ctx, w, bias, residual, gamma, beta),
                          test_utils=utils)
    w2 = (torch.randn(128, 128, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    torch.library.opcheck(B200.mlp_residual_layer_norm.default,
                          (ctx, w, bias, w2, bias, residual, gamma, beta), test_utils=utils)
    # the operators and the wrappers launch the same kernels: equal bits
    from solution.kernels import sm100_linear_residual_norm, sm100_mlp_residual_norm

    ln = torch.nn.LayerNorm(128).to(DEV)
    with torch.inference_mode():
        r_op, n_op = B200.linear_residual_layer_norm(ctx, w, bias, residual, ln.weight, ln.bias)
        r_w, n_w, _ = sm100_linear_residual_norm(ctx, w, bias, residual, ln, final_boundary=False)
        assert torch.equal(r_op, r_w) and torch.equal(n_op, n_w)
        r_op, n_op = B200.mlp_residual_layer_norm(ctx, w, bias, w2, bias, residual, ln.weight, ln.bias)
        r_w, n_w, _ = sm100_mlp_residual_norm(ctx, w, bias, w2, bias, residual, ln, final_boundary=False)
        assert torch.equal(r_op, r_w) and torch.equal(n_op, n_w)
