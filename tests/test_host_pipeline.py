"""HostPipeline: host batches through the forward with overlapped copies.

CPU tests cover argument checks.  The GPU tests check that pipelined results
are bit-identical to ``model(x.to(device))`` for a run of different batches
(so no slot is overwritten early and no output is read before its forward
finished) and that the overlap is real: the pipelined run takes less time
than the copies and forwards done one after another.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from oracle import OfficialConfig, official_input, official_state_dict
from solution import _native
from solution.runtimes.host_pipeline import HostPipeline
from solution.transformer import UserOptimizedTransformer, copy_model_weights


def test_depth_and_device_are_checked() -> None:
    with pytest.raises(ValueError):
        HostPipeline(lambda x: x, "cuda:0", depth=1)
    with pytest.raises(ValueError):
        HostPipeline(lambda x: x, "cuda:0", depth=True)
    with pytest.raises(RuntimeError):
        HostPipeline(lambda x: x, "cpu")


def _model(cfg: OfficialConfig) -> UserOptimizedTransformer:
    model = UserOptimizedTransformer(SimpleNamespace(**cfg.__dict__))
    copy_model_weights(official_state_dict(cfg, seed=0), model)
    return model.to("cuda:0").eval()


@pytest.mark.gpu
def test_pipelined_results_equal_plain_forward() -> None:
    cfg = OfficialConfig(4, 512, 256, 4, 1024, 2)
    model = _model(cfg)
    xs = [official_input(cfg, seed).pin_memory() for seed in range(5)]
    with torch.inference_mode():
        want = [model(x.to("cuda:0")).cpu() for x in xs]
    pipe = HostPipeline(model, "cuda:0", depth=2)
    outs = [torch.empty_like(x).pin_memory() for x in xs]
    with torch.inference_mode():
        got = pipe.run(xs, outs)
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert _native.device_error(clear=True) == 0


@pytest.mark.gpu
def test_host_buffers_must_be_pinned_and_shaped() -> None:
    cfg = OfficialConfig(1, 128, 256, 4, 1024, 1)
    model = _model(cfg)
    pipe = HostPipeline(model, "cuda:0")
    x = official_input(cfg, 0)
    with pytest.raises(ValueError, match="pinned"):
        pipe.submit(x, torch.empty_like(x).pin_memory())
    with pytest.raises(ValueError, match="out_host"):
        with torch.inference_mode():
            pipe.submit(x.pin_memory(), torch.empty(1, 64, 256).pin_memory())
    pipe.synchronize()


@pytest.mark.gpu
def test_copies_overlap_the_forward() -> None:
    cfg = OfficialConfig(8, 1024, 1024, 16, 4096, 2)
    model = _model(cfg)
    x = official_input(cfg, 1).pin_memory()
    outs = [torch.empty_like(x).pin_memory() for _ in range(2)]
    pipe = HostPipeline(model, "cuda:0")
    steps = 6
    with torch.inference_mode():
        for i in range(3):
            pipe.submit(x, outs[i % 2])
        pipe.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(pipe.copy_in)
        for i in range(steps):
            pipe.submit(x, outs[i % 2])
        end.record(pipe.copy_out)
        pipe.synchronize()
        pipelined = start.elapsed_time(end)

        # The same work done serially on one stream.
        x_dev = torch.empty_like(x, device="cuda:0")
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for i in range(steps):
            x_dev.copy_(x, non_blocking=True)
            outs[i % 2].copy_(model(x_dev), non_blocking=True)
        s1.record()
        torch.cuda.synchronize()
        serial = s0.elapsed_time(s1)
    assert pipelined < 0.9 * serial, (pipelined, serial)
