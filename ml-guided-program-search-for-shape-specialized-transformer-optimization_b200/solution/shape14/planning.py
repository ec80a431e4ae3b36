"""Legality of the streamed outer schedule.

Same rejection codes as the reference's streamed planning
(solution/shape14/planning.py:13-41) -- the codes and fields are the
interface that PlanBuilder's structured violations expose -- evaluated here
as a table of (condition, code, field, message) rules: every rule that holds
is reported, and the inner (per-microbatch) context is returned for the plan
of one microbatch.
"""

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
    """Report every violated streamed-schedule rule; return the microbatch context."""

    size = config.schedule.microbatch_size
    if size is None:
        raise RuntimeError("streamed configuration is missing its microbatch size")
    batch = context.batch_size
    rules = (
        (context.has_valid_token_mask, "mask_not_supported", "schedule.runtime",
         "the streamed schedule runs all-valid batches only (no valid_token_mask)"),
        (size > batch, "microbatch_exceeds_batch", "schedule.microbatch_size",
         f"microbatch of {size} rows is larger than the batch of {batch}"),
        (size <= batch and batch % size != 0, "microbatch_not_divisor", "schedule.microbatch_size",
         f"microbatch of {size} rows does not divide the batch of {batch}"),
    )
    for violated, code, field, message in rules:
        if violated:
            reject(code, field, message)
    return context.with_batch_size(size)


__all__ = ["validate_streamed_runtime"]
