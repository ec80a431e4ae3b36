"""Streamed execution: a long-sequence batch as microbatches written in place.

The reference runs its streamed (Shape-14) batch as ordered microbatches into
one preallocated output (solution/shape14/executor.py:12-49).  Here every
microbatch's forward writes its rows of the output itself: the program is
called as ``forward_chunk(chunk, mask_chunk, out=output_rows)``, where the
chunk and the output rows are contiguous views (batch rows are contiguous in
[B, S, D]).  Nothing is copied, and the activations of one microbatch are
released (back to the caching allocator) before the next one runs, which
bounds peak memory by one microbatch: about 2.6 GB per 100 000-token row at
D = 1024, F = 4096.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any

import torch

ChunkForward = Callable[..., Any]


def execute_streamed(
    value: torch.Tensor,
    valid_token_mask: torch.Tensor | None,
    *,
    microbatch_size: int,
    forward_chunk: ChunkForward,
    output: torch.Tensor | None = None,
) -> torch.Tensor:
    """Run ``value`` ([B, S, D]) as B / microbatch_size ordered microbatches.

    ``microbatch_size`` must divide B.  Returns ``output`` (allocated like
    ``value`` when not given), each microbatch's rows written by its own
    forward.
    """

    if isinstance(microbatch_size, bool) or not isinstance(microbatch_size, int) or microbatch_size <= 0:
        raise ValueError("microbatch_size must be a positive integer")
    batch = value.shape[0]
    if batch <= 0:
        raise ValueError("streamed execution requires a non-empty batch")
    if batch % microbatch_size:
        raise ValueError("microbatch_size must divide the batch size")
    if valid_token_mask is not None and valid_token_mask.shape[0] != batch:
        raise ValueError("valid_token_mask batch dimension must match the input")
    if not value.is_contiguous():
        raise ValueError("streamed execution reads contiguous batch rows")
    if output is None:
        output = torch.empty_like(value)
    elif output.shape != value.shape or not output.is_contiguous():
        raise ValueError("output must be a contiguous tensor of the input's shape")
    for start in range(0, batch, microbatch_size):
        rows = slice(start, start + microbatch_size)
        forward_chunk(
            value[rows], None if valid_token_mask is None else valid_token_mask[rows], out=output[rows]
        )
    return output


__all__ = ["execute_streamed"]
