"""Streamed capacity regime: ordered microbatches through the sm100 program.

Mirrors the reference's ``solution/shape14`` package (executor.py:12-49,
planning.py:13-41, defaults.py:22-49).  The reference needed a dedicated
Triton streaming kernel here; the sm100 flash-attention kernel already streams
KV tiles with its softmax state in registers at any sequence length, so this
package only holds the outer schedule.
"""

from .executor import execute_streamed
from .planning import validate_streamed_runtime

__all__ = ["execute_streamed", "validate_streamed_runtime"]
