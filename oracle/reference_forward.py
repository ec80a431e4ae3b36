"""numpy restatement of the reference Transformer forward -- TEST INFRASTRUCTURE.

Each function cites the reference line it restates
(official/torch_transformer_benchmark.py in the reference repository).  All
arithmetic is float32, as in the reference's CPU run; matrix products go
through numpy's BLAS.  Attention is evaluated in blocks of query rows so the
[S, S] score matrix is never held whole (the reference's own bounded-memory
equivalent is ``reference_causal_attention``,
solution/operators/attention/sdpa.py:116-170, pinned to the official op order
by tests/solution/test_causal_operators.py:62-83).
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf

EPS = 1e-5  # nn.LayerNorm default, official/torch_transformer_benchmark.py:128,130,160


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray, eps: float = EPS) -> np.ndarray:
    """nn.LayerNorm over the last axis: biased variance, eps inside the sqrt."""

    x = x.astype(np.float32, copy=False)
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float32)
    centred = x - mean
    var = (centred * centred).mean(axis=-1, keepdims=True, dtype=np.float32)
    return (centred / np.sqrt(var + np.float32(eps))) * weight + bias


def gelu_erf(x: np.ndarray) -> np.ndarray:
    """Exact GELU, F.gelu(approximate="none") (official :141)."""

    return (0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))).astype(np.float32)


def _linear(x: np.ndarray, weight: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """nn.Linear: x @ W^T + b."""

    return x @ weight.T + bias


def attention_reference(
    x: np.ndarray,
    state: dict[str, np.ndarray],
    prefix: str,
    num_heads: int,
    causal: bool,
    valid_token_mask: np.ndarray | None = None,
    query_block: int = 256,
) -> np.ndarray:
    """BaselineSelfAttention.forward (official :86-122) for x of shape [B, S, D].

    q/k/v projections, heads split [B, H, S, Dh], scores = q k^T * Dh^-1/2,
    causal positions above the diagonal -> -inf (:99-103), invalid keys -> -inf
    (:105-108), softmax in fp32 (:111), probs @ v, heads merged, out_proj, then
    invalid query rows zeroed (:120-121).
    """

    batch, seq, d_model = x.shape
    head_dim = d_model // num_heads
    scale = np.float32(head_dim**-0.5)

    def heads(t: np.ndarray) -> np.ndarray:
        return t.reshape(batch, seq, num_heads, head_dim).transpose(0, 2, 1, 3)

    q = heads(_linear(x, state[f"{prefix}.q_proj.weight"], state[f"{prefix}.q_proj.bias"]))
    k = heads(_linear(x, state[f"{prefix}.k_proj.weight"], state[f"{prefix}.k_proj.bias"]))
    v = heads(_linear(x, state[f"{prefix}.v_proj.weight"], state[f"{prefix}.v_proj.bias"]))
    context = np.empty((batch, num_heads, seq, head_dim), dtype=np.float32)
    key_pos = np.arange(seq)
    for start in range(0, seq, query_block):
        stop = min(start + query_block, seq)
        scores = np.matmul(q[:, :, start:stop], k.transpose(0, 1, 3, 2)) * scale
        if causal:
            above = key_pos[None, :] > np.arange(start, stop)[:, None]
            scores = np.where(above[None, None], np.float32(-np.inf), scores)
        if valid_token_mask is not None:
            scores = np.where(~valid_token_mask[:, None, None, :], np.float32(-np.inf), scores)
        scores = scores - scores.max(axis=-1, keepdims=True)
        probs = np.exp(scores, dtype=np.float32)
        probs /= probs.sum(axis=-1, keepdims=True)
        context[:, :, start:stop] = np.matmul(probs, v)
    merged = context.transpose(0, 2, 1, 3).reshape(batch, seq, d_model)
    out = _linear(merged, state[f"{prefix}.out_proj.weight"], state[f"{prefix}.out_proj.bias"])
    if valid_token_mask is not None:
        out = np.where(valid_token_mask[..., None], out, np.float32(0.0))
    return out.astype(np.float32, copy=False)


def attention_core(
    q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool, query_block: int = 256
) -> np.ndarray:
    """softmax(q k^T * Dh^-1/2 [+ causal -inf]) v for [B, H, S, Dh] float32 arrays.

    The score/softmax/PV core of official :97-112 without the projections.
    """

    batch, heads, seq, head_dim = q.shape
    scale = np.float32(head_dim**-0.5)
    out = np.empty_like(q, dtype=np.float32)
    key_pos = np.arange(k.shape[2])
    for start in range(0, seq, query_block):
        stop = min(start + query_block, seq)
        scores = np.matmul(q[:, :, start:stop], k.transpose(0, 1, 3, 2)) * scale
        if causal:
            above = key_pos[None, :] > np.arange(start, stop)[:, None]
            scores = np.where(above[None, None], np.float32(-np.inf), scores)
        scores = scores - scores.max(axis=-1, keepdims=True)
        probs = np.exp(scores, dtype=np.float32)
        probs /= probs.sum(axis=-1, keepdims=True)
        out[:, :, start:stop] = np.matmul(probs, v)
    return out


def ffn_reference(x: np.ndarray, state: dict[str, np.ndarray], prefix: str) -> np.ndarray:
    """ffn_out(GELU(ffn_in(x))) (official :141)."""

    hidden = gelu_erf(_linear(x, state[f"{prefix}.ffn_in.weight"], state[f"{prefix}.ffn_in.bias"]))
    return _linear(hidden, state[f"{prefix}.ffn_out.weight"], state[f"{prefix}.ffn_out.bias"])


def transformer_forward(
    x: np.ndarray,
    state: dict[str, np.ndarray],
    *,
    num_heads: int,
    num_layers: int,
    causal: bool = True,
    valid_token_mask: np.ndarray | None = None,
    query_block: int = 256,
) -> np.ndarray:
    """BaselineTransformer.forward (official :148-172) on a [B, S, D] float32 input.

    Per block (official :136-145): x += attention(LN1(x)); x += FFN(LN2(x));
    invalid rows zeroed after each block; final LayerNorm; invalid rows zeroed.
    ``state`` uses the official parameter names (``layers.{i}.attention.q_proj.weight``).
    """

    x = np.asarray(x, dtype=np.float32)
    for i in range(num_layers):
        p = f"layers.{i}"
        normed = layer_norm(x, state[f"{p}.norm1.weight"], state[f"{p}.norm1.bias"])
        x = x + attention_reference(
            normed, state, f"{p}.attention", num_heads, causal, valid_token_mask, query_block
        )
        normed = layer_norm(x, state[f"{p}.norm2.weight"], state[f"{p}.norm2.bias"])
        x = x + ffn_reference(normed, state, p)
        if valid_token_mask is not None:
            x = np.where(valid_token_mask[..., None], x, np.float32(0.0))
    y = layer_norm(x, state["final_norm.weight"], state["final_norm.bias"])
    if valid_token_mask is not None:
        y = np.where(valid_token_mask[..., None], y, np.float32(0.0))
    return y.astype(np.float32, copy=False)


__all__ = [
    "EPS",
    "attention_core",
    "attention_reference",
    "ffn_reference",
    "gelu_erf",
    "layer_norm",
    "transformer_forward",
]
