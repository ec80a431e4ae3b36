"""Host-resident batches through the sm100 forward with copies overlapped.

The reference's callers hand the model a device tensor and read the result
back themselves (official/torch_transformer_benchmark.py:486-500); between
batches the GPU idles while PCIe moves the next input and the last output.
``HostPipeline`` takes batches that live in pinned host memory and keeps three
CUDA streams busy at once:

    copy-in stream   H2D of batch i+1 into device slot (i+1) % depth
    compute stream   forward of batch i (every libb200tx launch of the plan)
    copy-out stream  D2H of batch i-1's output into the caller's host buffer

Ordering is carried by CUDA events only (no host synchronisation inside
``submit``):

* the copy into slot s waits until the forward that last read slot s is done;
* the forward of batch i waits for its copy-in;
* the copy-out of batch i waits for its forward, and the output tensor is
  marked as used by the copy-out stream so the caching allocator cannot hand
  its memory to a later forward before the copy has read it.

Results are bit-identical to ``model(x.to(device))``: the same program runs on
the same data, only on another stream.  The caller owns the pinned host
buffers; a result may be read after its handle's ``wait()``.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass

import torch

Forward = Callable[[torch.Tensor], torch.Tensor]


@dataclass
class PipelineHandle:
    """One submitted batch: its host output and the event that completes it."""

    output: torch.Tensor
    done: torch.cuda.Event

    def ready(self) -> bool:
        return self.done.query()

    def wait(self) -> torch.Tensor:
        self.done.synchronize()
        return self.output


class HostPipeline:
    """Overlap H2D copy, forward and D2H copy across consecutive host batches.

    ``forward`` is any callable mapping a device ``[B, S, D]`` tensor to a
    device tensor (a ``UserOptimizedTransformer`` or a sharded wrapper);
    ``depth`` device input slots (>= 2) bound how far copy-in runs ahead.
    """

    def __init__(self, forward: Forward, device: torch.device | str, *, depth: int = 2) -> None:
        if isinstance(depth, bool) or not isinstance(depth, int) or depth < 2:
            raise ValueError("depth must be an integer >= 2")
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("HostPipeline runs on CUDA devices only")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.forward = forward
        self.device = device
        self.depth = depth
        self.copy_in = torch.cuda.Stream(device)
        self.compute = torch.cuda.Stream(device)
        self.copy_out = torch.cuda.Stream(device)
        self._slots: list[torch.Tensor | None] = [None] * depth
        self._slot_free: list[torch.cuda.Event | None] = [None] * depth
        self._submitted = 0

    def _slot(self, index: int, like: torch.Tensor) -> torch.Tensor:
        slot = self._slots[index]
        if slot is None or slot.shape != like.shape or slot.dtype != like.dtype:
            if slot is not None:
                # Reallocating: the previous buffer must no longer be read.
                free = self._slot_free[index]
                if free is not None:
                    free.synchronize()
            with torch.cuda.device(self.device):
                slot = torch.empty(like.shape, dtype=like.dtype, device=self.device)
            self._slots[index] = slot
        return slot

    def submit(self, x_host: torch.Tensor, out_host: torch.Tensor) -> PipelineHandle:
        """Queue one batch; returns at once with a handle for its result."""

        if x_host.device.type != "cpu" or out_host.device.type != "cpu":
            raise ValueError("x_host and out_host must be host tensors")
        if not (x_host.is_pinned() and out_host.is_pinned()):
            raise ValueError("x_host and out_host must be in pinned memory (tensor.pin_memory())")
        if not x_host.is_contiguous() or not out_host.is_contiguous():
            raise ValueError("x_host and out_host must be contiguous")
        index = self._submitted % self.depth
        slot = self._slot(index, x_host)

        loaded = torch.cuda.Event()
        with torch.cuda.stream(self.copy_in):
            free = self._slot_free[index]
            if free is not None:
                self.copy_in.wait_event(free)
            slot.copy_(x_host, non_blocking=True)
            loaded.record(self.copy_in)

        computed = torch.cuda.Event()
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(loaded)
            y = self.forward(slot)
            computed.record(self.compute)
        self._slot_free[index] = computed
        if y.shape != out_host.shape or y.dtype != out_host.dtype:
            raise ValueError(
                f"out_host must be {tuple(y.shape)} {y.dtype}, got {tuple(out_host.shape)} {out_host.dtype}"
            )
        y.record_stream(self.copy_out)

        done = torch.cuda.Event()
        with torch.cuda.stream(self.copy_out):
            self.copy_out.wait_event(computed)
            out_host.copy_(y, non_blocking=True)
            done.record(self.copy_out)
        self._submitted += 1
        return PipelineHandle(output=out_host, done=done)

    def run(self, batches: Iterable[torch.Tensor], outputs: Sequence[torch.Tensor]) -> list[torch.Tensor]:
        """Submit every batch into its output buffer, then wait for all."""

        handles = [self.submit(x, out) for x, out in zip(batches, outputs, strict=True)]
        return [h.wait() for h in handles]

    def synchronize(self) -> None:
        for stream in (self.copy_in, self.compute, self.copy_out):
            stream.synchronize()


__all__ = ["HostPipeline", "PipelineHandle"]
