"""Outer execution schedules over the sm100 kernels.

Mirrors the reference's ``solution/runtimes`` (cuda_graph.py:11-141,
batch_tiled_graph.py:10-127).  ``torch.compile`` schedules are not offered.
"""

from .batch_tiled_graph import BatchTiledGraphReplay
from .cuda_graph import CudaGraphReplay

__all__ = ["BatchTiledGraphReplay", "CudaGraphReplay"]
