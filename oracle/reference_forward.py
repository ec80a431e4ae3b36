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


def attention_rows(
    q: np.ndarray, k: np.ndarray, v: np.ndarray, query_rows: np.ndarray, causal: bool = True
) -> np.ndarray:
    """The score/softmax/PV core of official :97-112 for selected query rows of one head.

    ``k``, ``v`` are [S, Dh] float32 arrays of one (batch, head); ``q`` holds
    the queries of the rows whose absolute positions are ``query_rows``
    ([len(query_rows), Dh]).  Each row attends to the keys at positions <= its
    own (causal) or to all keys.  The cost is
    len(query_rows) x S x Dh, so a few rows of an S = 100 000 sequence are
    checked in well under a second.
    """

    rows = np.asarray(query_rows, dtype=np.int64)
    scale = np.float32(q.shape[-1] ** -0.5)
    scores = (q @ k.T) * scale
    if causal:
        above = np.arange(k.shape[0])[None, :] > rows[:, None]
        scores = np.where(above, np.float32(-np.inf), scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    probs = np.exp(scores, dtype=np.float32)
    probs /= probs.sum(axis=-1, keepdims=True)
    return (probs @ v).astype(np.float32, copy=False)


def _threaded_causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, query_block: int = 512) -> np.ndarray:
    """attention_core for [H, S, Dh] arrays, causal, one head per worker thread.

    Query block [a, b) only multiplies against keys [0, b): the keys above the
    block's last row are masked to -inf by the reference and contribute exact
    zeros, so leaving them out changes no value.  numpy releases the GIL in
    its BLAS calls and ufuncs, so the heads run in parallel on the host cores.
    """

    import os
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    heads, seq, head_dim = q.shape
    scale = np.float32(head_dim**-0.5)
    out = np.empty_like(q, dtype=np.float32)

    def one_head(h: int) -> None:
        for start in range(0, seq, query_block):
            stop = min(start + query_block, seq)
            scores = (q[h, start:stop] @ k[h, :stop].T) * scale
            above = np.arange(stop)[None, :] > np.arange(start, stop)[:, None]
            scores = np.where(above, np.float32(-np.inf), scores)
            scores -= scores.max(axis=-1, keepdims=True)
            probs = np.exp(scores, dtype=np.float32)
            probs /= probs.sum(axis=-1, keepdims=True)
            out[h, start:stop] = probs @ v[h, :stop]

    with threadpool_limits(1), ThreadPoolExecutor(max_workers=min(heads, os.cpu_count() or 1)) as pool:
        list(pool.map(one_head, range(heads)))
    return out


def transformer_forward_tail(
    x: np.ndarray,
    state: dict[str, np.ndarray],
    *,
    num_heads: int,
    num_layers: int,
    tail: int,
) -> np.ndarray:
    """The last ``tail`` positions of BaselineTransformer.forward (official
    :148-172, causal, no mask) for ONE batch row x of shape [1, S, D].

    Every layer but the last runs on all S positions (the next layer's keys
    and values depend on all of them).  In the last layer only the keys and
    values are computed for all positions; the queries, attention rows,
    out-projection, FFN and final LayerNorm run on the last ``tail`` rows,
    whose values do not depend on the other rows' outputs of that layer.
    Same operations in the same order as transformer_forward, so the result
    equals transformer_forward(x)[:, -tail:] up to BLAS summation order.
    """

    x = np.asarray(x, dtype=np.float32)[0]
    seq, d_model = x.shape
    head_dim = d_model // num_heads

    def split(t: np.ndarray) -> np.ndarray:
        return np.ascontiguousarray(t.reshape(t.shape[0], num_heads, head_dim).transpose(1, 0, 2))

    for i in range(num_layers):
        p = f"layers.{i}"
        a = f"{p}.attention"
        normed = layer_norm(x, state[f"{p}.norm1.weight"], state[f"{p}.norm1.bias"])
        k = split(_linear(normed, state[f"{a}.k_proj.weight"], state[f"{a}.k_proj.bias"]))
        v = split(_linear(normed, state[f"{a}.v_proj.weight"], state[f"{a}.v_proj.bias"]))
        if i < num_layers - 1:
            q = split(_linear(normed, state[f"{a}.q_proj.weight"], state[f"{a}.q_proj.bias"]))
            context = _threaded_causal_attention(q, k, v)
        else:
            rows = np.arange(seq - tail, seq)
            x = x[rows]
            q = split(_linear(normed[rows], state[f"{a}.q_proj.weight"], state[f"{a}.q_proj.bias"]))
            context = np.stack([attention_rows(q[h], k[h], v[h], rows) for h in range(num_heads)])
        merged = context.transpose(1, 0, 2).reshape(-1, d_model)
        x = x + _linear(merged, state[f"{a}.out_proj.weight"], state[f"{a}.out_proj.bias"])
        normed = layer_norm(x, state[f"{p}.norm2.weight"], state[f"{p}.norm2.bias"])
        x = x + ffn_reference(normed, state, p)
    return layer_norm(x, state["final_norm.weight"], state["final_norm.bias"]).astype(np.float32, copy=False)


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
    "attention_rows",
    "attention_reference",
    "ffn_reference",
    "gelu_erf",
    "layer_norm",
    "transformer_forward",
    "transformer_forward_tail",
]
