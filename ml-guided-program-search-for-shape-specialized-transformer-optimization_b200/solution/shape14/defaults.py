"""Default streamed program for the capacity shape.

The reference pins a conservative streamed default for its Shape 14
(solution/shape14/defaults.py:22-49: B32/S100000/D1024/H16/L2, microbatch 2).
The sm100 program keeps all activations of a microbatch resident; one batch
row at S=100 000, D=1024, F=4096 needs about 2.6 GB of activations, so the
default microbatch is 4 rows (about 10 GB), well inside 180 GB of HBM while
keeping each launch large enough to fill 148 SMs.
"""

from __future__ import annotations

from ..config import ConfigSpec, portable_streamed_config

STREAMED_DEFAULT_MICROBATCH = 4


def default_streamed_config(batch_size: int) -> ConfigSpec:
    """Largest divisor of the batch not above the default microbatch."""

    microbatch = 1
    for candidate in range(min(batch_size, STREAMED_DEFAULT_MICROBATCH), 0, -1):
        if batch_size % candidate == 0:
            microbatch = candidate
            break
    return portable_streamed_config(microbatch_size=microbatch)


def is_streamed_shape(seq_len: int, d_model: int) -> bool:
    """Shapes whose activations are streamed by default (S >= 65 536)."""

    return seq_len >= 65536 and d_model >= 512


__all__ = ["STREAMED_DEFAULT_MICROBATCH", "default_streamed_config", "is_streamed_shape"]
