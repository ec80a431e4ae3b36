"""Outer execution schedules over the sm100 kernels.

Mirrors the reference's ``solution/runtimes`` (cuda_graph.py:11-141,
batch_tiled_graph.py:10-127).  ``torch.compile`` schedules are not offered.
Added for B200: ``HostPipeline`` (host batches with copies overlapped on
separate streams), ``sharded`` (batch- and head-sharded multi-GPU forward) and
``liveness`` (host-side detection of a failed rank between steps).
"""

from .batch_tiled_graph import BatchTiledGraphReplay
from .cuda_graph import CudaGraphReplay
from .host_pipeline import HostPipeline, PipelineHandle
from .liveness import RankFailure, StepLiveness, abort_process_group

__all__ = [
    "BatchTiledGraphReplay",
    "CudaGraphReplay",
    "HostPipeline",
    "PipelineHandle",
    "RankFailure",
    "StepLiveness",
    "abort_process_group",
]
