"""Streamed-runtime validation (reference: solution/shape14/planning.py:13-41)."""

from __future__ import annotations

from collections.abc import Callable

from ..config import ConfigSpec
from ..plan import ExecutionContext

Reject = Callable[[str, str, str], None]


def validate_streamed_runtime(
    config: ConfigSpec,
    context: ExecutionContext,
    reject: Reject,
) -> ExecutionContext:
    """Validate the streamed outer schedule and return its inner context."""

    microbatch_size = config.schedule.microbatch_size
    if microbatch_size is None:
        raise RuntimeError("streamed configuration is missing its microbatch size")
    if context.has_valid_token_mask:
        reject(
            "mask_not_supported",
            "schedule.runtime",
            "streamed execution requires an all-valid workload",
        )
    if microbatch_size > context.batch_size:
        reject(
            "microbatch_exceeds_batch",
            "schedule.microbatch_size",
            "microbatch cannot exceed the logical batch",
        )
    elif context.batch_size % microbatch_size:
        reject(
            "microbatch_not_divisor",
            "schedule.microbatch_size",
            "microbatch must divide the logical batch",
        )
    return context.with_batch_size(microbatch_size)


__all__ = ["validate_streamed_runtime"]
