"""Batch-tiled CUDA-graph replay over slices of the caller's own input.

Batch rows are independent in every operator of the block, so a batch can
run as consecutive tiles of ``tile_size`` rows (the reference's
``BatchTiledGraphReplay``, solution/runtimes/batch_tiled_graph.py:10-127,
replays one graph over tiles staged through a static buffer, zero-padding the
last one).  Here each tile of a bound input is its own capture, made on the
tile's slice of the caller's tensor (rows are contiguous in [B, S, D], so a
tile is a view, never a copy); a short last tile is captured at its own size,
so nothing is padded or computed twice.  After each tile's replay its final
launch (see ``cuda_graph``) writes the tile's rows of the call's output
directly.

All tile captures of all bindings share one graph memory pool.  A tile's
replay and its final launch run back to back on one stream, and the buffers
that final launch reads stay allocated for the binding's lifetime, so the
shared pool holds one tile's transient activations plus each tile's small
set of live buffers, and no replay overwrites another tile's live buffers.
"""

from __future__ import annotations

from collections import OrderedDict
from collections.abc import Callable

import torch

from .cuda_graph import Program, capture_program


class BatchTiledGraphReplay:
    """Run independent batch tiles of a bound input through per-tile graphs."""

    def __init__(self, tile_size: int, *, max_bindings: int = 2) -> None:
        if isinstance(tile_size, bool) or not isinstance(tile_size, int):
            raise TypeError("tile_size must be an integer")
        if tile_size <= 0:
            raise ValueError("tile_size must be positive")
        if max_bindings < 1:
            raise ValueError("max_bindings must be at least 1")
        self._tile_size = tile_size
        self.max_bindings = max_bindings
        # key -> (held input, [(rows, graph, finish), ...])
        self._bindings: OrderedDict[
            tuple[object, ...],
            tuple[torch.Tensor, list[tuple[slice, torch.cuda.CUDAGraph, Callable[[torch.Tensor], torch.Tensor]]]],
        ] = OrderedDict()
        self._layout: tuple[object, ...] | None = None
        self._pool: object | None = None

    @property
    def tile_size(self) -> int:
        return self._tile_size

    @property
    def captured(self) -> bool:
        return bool(self._bindings)

    def _bind(self, program: Program, value: torch.Tensor) -> list:
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        tiles = []
        for start in range(0, value.shape[0], self._tile_size):
            rows = slice(start, min(start + self._tile_size, value.shape[0]))
            graph, finish = capture_program(program, value[rows], None, self._pool)
            tiles.append((rows, graph, finish))
        return tiles

    def run(self, program: Program, value: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
        """Replay every tile of ``value`` (capturing on first use) into one fresh output."""

        if value.device.type != "cuda":
            raise ValueError("batch-tiled CUDA graph requires a CUDA input")
        if value.ndim != 3 or not value.is_contiguous():
            raise ValueError("batch-tiled CUDA graph requires a contiguous 3D input")
        if value.shape[0] <= self._tile_size:
            raise ValueError("batch-tiled CUDA graph requires more than one tile")
        if mask is not None:
            raise ValueError("batch-tiled CUDA graph does not accept a token mask")
        layout = (value.device, value.dtype, tuple(value.shape))
        if self._layout is not None and layout != self._layout:
            raise RuntimeError("batch-tiled CUDA graph supports one full input signature")
        key = (value.data_ptr(), layout)
        entry = self._bindings.get(key)
        if entry is None:
            tiles = self._bind(program, value)
            if len(self._bindings) >= self.max_bindings:
                self._bindings.popitem(last=False)
            entry = (value, tiles)
            self._bindings[key] = entry
            self._layout = layout
        else:
            self._bindings.move_to_end(key)
        output = torch.empty_like(value)
        for rows, graph, finish in entry[1]:
            graph.replay()
            finish(output[rows])
        return output

    def release(self) -> None:
        self._bindings.clear()
        self._layout = None
        self._pool = None


__all__ = ["BatchTiledGraphReplay"]
