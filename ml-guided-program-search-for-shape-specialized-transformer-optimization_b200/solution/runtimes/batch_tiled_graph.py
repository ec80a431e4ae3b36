"""Batch-tiled execution through one fixed-shape CUDA graph.

Same contract as the reference's ``BatchTiledGraphReplay``
(solution/runtimes/batch_tiled_graph.py:10-127): batch rows are independent in
every operator of the block, so one graph captured for ``tile_size`` rows is
replayed over consecutive tiles of the logical batch; a short tail tile is
zero-padded and only its valid rows are copied out.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

Forward = Callable[[torch.Tensor, None], torch.Tensor]


class BatchTiledGraphReplay:
    """Run independent batch tiles through one captured forward graph."""

    def __init__(self, tile_size: int) -> None:
        if isinstance(tile_size, bool) or not isinstance(tile_size, int):
            raise TypeError("tile_size must be an integer")
        if tile_size <= 0:
            raise ValueError("tile_size must be positive")
        self._tile_size = tile_size
        self._signature: tuple[object, ...] | None = None
        self._graph: torch.cuda.CUDAGraph | None = None
        self._static_input: torch.Tensor | None = None
        self._static_output: torch.Tensor | None = None

    @property
    def tile_size(self) -> int:
        return self._tile_size

    @staticmethod
    def _sig(value: torch.Tensor) -> tuple[object, ...]:
        return (value.device, value.dtype, tuple(value.shape), tuple(value.stride()))

    def _capture(self, function: Forward, value: torch.Tensor) -> None:
        static_input = torch.zeros(
            (self._tile_size, *value.shape[1:]), device=value.device, dtype=value.dtype
        )
        first = min(value.shape[0], self._tile_size)
        static_input[:first].copy_(value[:first])
        current = torch.cuda.current_stream(value.device)
        side = torch.cuda.Stream(device=value.device)
        side.wait_stream(current)
        with torch.cuda.stream(side), torch.inference_mode():
            for _ in range(3):
                function(static_input, None)
        current.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(graph, stream=side):
            static_output = function(static_input, None)
        current.wait_stream(side)
        if not isinstance(static_output, torch.Tensor):
            raise TypeError("batch-tiled graph function must return a Tensor")
        if static_output.shape != static_input.shape:
            raise RuntimeError("batch-tiled graph output shape must match its input")
        if static_output.device != value.device or static_output.dtype != value.dtype:
            raise RuntimeError("batch-tiled graph output must keep the input device and dtype")
        self._signature = self._sig(value)
        self._graph = graph
        self._static_input = static_input
        self._static_output = static_output

    def run(self, function: Forward, value: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
        """Replay every tile and assemble one independent full output."""

        if value.device.type != "cuda":
            raise ValueError("batch-tiled CUDA graph requires a CUDA input")
        if value.ndim != 3 or not value.is_contiguous():
            raise ValueError("batch-tiled CUDA graph requires a contiguous 3D input")
        if value.shape[0] <= self._tile_size:
            raise ValueError("batch-tiled CUDA graph requires more than one tile")
        if mask is not None:
            raise ValueError("batch-tiled CUDA graph does not accept a token mask")
        signature = self._sig(value)
        if self._graph is not None and signature != self._signature:
            raise RuntimeError("batch-tiled CUDA graph supports one full input signature")
        if self._graph is None:
            self._capture(function, value)
        assert self._graph is not None and self._static_input is not None
        assert self._static_output is not None
        output = torch.empty_like(value)
        for start in range(0, value.shape[0], self._tile_size):
            stop = min(start + self._tile_size, value.shape[0])
            count = stop - start
            if count == self._tile_size:
                self._static_input.copy_(value[start:stop])
            else:
                self._static_input.zero_()
                self._static_input[:count].copy_(value[start:stop])
            self._graph.replay()
            output[start:stop].copy_(self._static_output[:count])
        return output

    def release(self) -> None:
        self._graph = None
        self._static_input = None
        self._static_output = None
        self._signature = None


__all__ = ["BatchTiledGraphReplay"]
