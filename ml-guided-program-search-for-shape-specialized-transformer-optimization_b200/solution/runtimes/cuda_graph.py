"""CUDA-graph replay of the forward, bound to the caller's own buffers.

The graph runtime of the reference (``CudaGraphReplay``,
solution/runtimes/cuda_graph.py:11-141) stages every input into a static
buffer and clones the static output.  Here a graph is captured per *input
buffer* instead:

* the captured kernels read the caller's input tensor where it lies, so no
  input is copied;
* the pass's last launch -- the final LayerNorm (or the fused boundary that
  ends the last block), the only kernel that writes the output -- is kept out
  of the graph and launched after each replay straight into the output tensor
  allocated for that call, so nothing is copied out either.

A call is one graph launch plus one kernel launch, and moves no bytes beyond
the forward's own.  At the C2 shape that removes a 64 MB copy in and a 64 MB
clone out (about 40 us of a 1 ms step) and all per-kernel host work.

Bindings.  A binding is keyed by the data pointers, shapes, strides and
dtypes of the input and mask.  It holds references to those tensors, so their
storage cannot be freed and handed to another tensor while a graph that reads
it exists.  Up to ``max_bindings`` bindings are kept, least recently used
dropped first.  Their intermediates come from one graph memory pool: every
replay and its final launch run back to back on one stream, and the buffers a
binding's final launch reads stay allocated for the binding's lifetime, so no
replay can overwrite another binding's live buffers.  Values are read at
replay time: changing the bound input in place between calls is seen by the
next call, as with the eager forward.

Every binding has the shape of the first one (the model's plan is built per
input signature); another shape is rejected.
"""

from __future__ import annotations

from collections import OrderedDict
from collections.abc import Callable
from typing import Any

import torch

# program(value, mask, *, out=None, defer_final=False): the model's planned
# forward.  With defer_final it launches everything but the last kernel and
# returns finish(out), which launches that kernel into ``out`` and returns it.
Program = Callable[..., Any]


def _layout(t: torch.Tensor | None) -> tuple[object, ...] | None:
    if t is None:
        return None
    return (t.device, t.dtype, tuple(t.shape), tuple(t.stride()))


class _Binding:
    __slots__ = ("finish", "graph", "tensors")

    def __init__(self, graph: torch.cuda.CUDAGraph, finish: Callable[[torch.Tensor], torch.Tensor],
                 tensors: tuple[torch.Tensor, torch.Tensor | None]) -> None:
        self.graph = graph
        self.finish = finish
        self.tensors = tensors


def capture_program(
    program: Program, value: torch.Tensor, mask: torch.Tensor | None, pool: object
) -> tuple[torch.cuda.CUDAGraph, Callable[[torch.Tensor], torch.Tensor]]:
    """Capture ``program`` on ``value``/``mask`` in place; return the graph and
    the deferred final launch.  One eager run on the capture stream first
    completes every lazy set-up of the launches (weight shadows, kernel
    attributes, the tensor-map encoder), none of which may happen inside a
    capture."""

    device = value.device
    current = torch.cuda.current_stream(device)
    side = torch.cuda.Stream(device=device)
    side.wait_stream(current)
    with torch.cuda.stream(side), torch.inference_mode():
        program(value, mask)
    graph = torch.cuda.CUDAGraph()
    with torch.inference_mode(), torch.cuda.graph(graph, pool=pool, stream=side):
        finish = program(value, mask, defer_final=True)
    current.wait_stream(side)
    return graph, finish


class CudaGraphReplay:
    """Graph replays of one input signature, one capture per bound buffer."""

    def __init__(self, *, reuse_unchanged_input: bool = False, max_bindings: int = 4) -> None:
        # ``reuse_unchanged_input`` is the schedule knob of the reference's
        # staging copy; with the input bound in place no call copies it, so
        # the knob has nothing left to skip and is accepted as is.
        if max_bindings < 1:
            raise ValueError("max_bindings must be at least 1")
        self.reuse_unchanged_input = reuse_unchanged_input
        self.max_bindings = max_bindings
        self._bindings: OrderedDict[tuple[object, ...], _Binding] = OrderedDict()
        self._layout: tuple[object, ...] | None = None
        self._pool: object | None = None

    @property
    def captured(self) -> bool:
        return bool(self._bindings)

    @property
    def bindings(self) -> int:
        return len(self._bindings)

    def run(self, program: Program, value: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
        """Replay the graph bound to ``value`` (capturing it on first use) and
        write a fresh output."""

        layout = (_layout(value), _layout(mask))
        if self._layout is not None and layout != self._layout:
            raise RuntimeError(
                "CUDA graph replay supports one static input signature per model; "
                "create or reconfigure the model for a different signature"
            )
        key = (value.data_ptr(), None if mask is None else mask.data_ptr(), layout)
        binding = self._bindings.get(key)
        if binding is None:
            if self._pool is None:
                self._pool = torch.cuda.graph_pool_handle()
            graph, finish = capture_program(program, value, mask, self._pool)
            if len(self._bindings) >= self.max_bindings:
                self._bindings.popitem(last=False)
            binding = _Binding(graph, finish, (value, mask))
            self._bindings[key] = binding
            self._layout = layout
        else:
            self._bindings.move_to_end(key)
        binding.graph.replay()
        return binding.finish(torch.empty_like(value, memory_format=torch.contiguous_format))

    def release(self) -> None:
        """Drop every binding (graphs, their buffers and the held inputs)."""

        self._bindings.clear()
        self._layout = None
        self._pool = None


__all__ = ["CudaGraphReplay", "Program", "capture_program"]
