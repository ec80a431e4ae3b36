#!/usr/bin/env python3
"""Forward-throughput benchmark of the sm_100a Transformer (one JSON line).

Workload (N=1): BASELINE config C2 -- B=8, S=2048, D=1024, 16 heads
(head_dim 64), 2 layers, causal, FFN 4096 exact GELU; x ~ N(0,1) from seed 1,
weights = the reference module's seeded default init (seed 0).  A "step" is
one full forward over that batch.  Under torchrun each rank runs its own C2
batch (batch sharding, no collective): per-GPU work is fixed, ``scaling`` is
"weak" and ``value`` is the total tokens/s of all ranks over the slowest
rank's time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

``value``      tokens/s with x already in HBM, each step bracketed by CUDA
               events on the launching stream, L2 flushed before every step.
``e2e``        tokens/s through the public host-batch API (HostPipeline) with x
               in pinned host memory: H2D copy of x, forward, D2H copy of the
               whole output, every step, on three overlapping CUDA streams.
``roofline``   the dominant kernel (by time) of the step, timed live with
               CUDA events around its launches; peak = the measured burst
               bf16 GEMM rate (tensor-bound) or copy bandwidth (HBM-bound).
``workloads``  the other BASELINE configs on the same N GPUs, each with its
               own ms_per_step, clocks and peak memory: C3 (batch-sharded,
               weak), C4 (1 GPU, else head-sharded tp2 groups x batch
               replicas), C5 (the 32 x 100 000-token rows split over the
               ranks, streamed).
``tp_parity``  (N >= 2) the head-sharded forward (NCCL and peer-memory
               reductions) against the reference's CPU forward.
``cpu_baseline`` the reference's own PyTorch CPU forward
               (official.BaselineTransformer, installed in baseline/_ref) on
               one batch row, on all host cores; ``reference_parity`` compares
               this run's GPU output row with it.  Without the install, the
               numpy restatement in oracle/ (kind "port").
``--impl reference`` times that CPU forward alone, as the reference arm.
``--kernel NAME`` times one libb200tx kernel alone on its C2-shaped operands
               (attention, qkv, out_proj, ffn_in, ffn_out, residual_norm) and
               prints its own JSON line; ncu profiles in profiles/ use this mode.
``--workload official`` times the reference's own benchmark table (its 14
               official shapes) under the eager and CUDA-graph schedules and
               prints one JSON line with the reference's published medians
               beside each shape.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path
from types import SimpleNamespace

REPO = Path(__file__).resolve().parent
PACKAGE_DIR = REPO / "ml-guided-program-search-for-shape-specialized-transformer-optimization_b200"
for _p in (str(PACKAGE_DIR), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

WORKLOAD = dict(batch_size=8, seq_len=2048, d_model=1024, num_heads=16, ffn_dim=4096, num_layers=2, causal=True)
# BASELINE.json configs run by --workload (c2 is the default bench line).
WORKLOADS = {
    "c2": (WORKLOAD, 1, "C2 resident mid shape: B8 S2048 D1024 H16(Dh64) F4096 L2 causal"),
    "c3": (dict(batch_size=64, seq_len=256, d_model=768, num_heads=12, ffn_dim=3072, num_layers=4, causal=True), 2,
           "C3 short-sequence large-batch: B64 S256 D768 H12(Dh64) F3072 L4 causal"),
    "c4": (dict(batch_size=4, seq_len=16384, d_model=2048, num_heads=32, ffn_dim=8192, num_layers=2, causal=True), 3,
           "C4 long-context: B4 S16384 D2048 H32(Dh64) F8192 L2 causal"),
    "c5": (dict(batch_size=32, seq_len=100000, d_model=1024, num_heads=16, ffn_dim=4096, num_layers=2, causal=True), 4,
           "C5 streamed capacity: B32 S100000 D1024 H16(Dh64) F4096 L2 causal"),
}
INPUT_SEED = 1
WEIGHT_SEED = 0
METRIC = "fwd tokens/s"
UNIT = "tokens/s"
WORKLOAD_NAME = "C2 resident mid shape: B8 S2048 D1024 H16(Dh64) F4096 L2 causal"
L2_FLUSH_BYTES = 256 * 1024 * 1024
L2_FLUSH_NOTE = "flushed before every timed step (256 MB written, then 256 MB of another buffer read)"


class L2Flush:
    """Evict the L2 between timed steps without leaving write-backs behind.

    Writing a buffer larger than the L2 (126 MB) evicts the step's inputs, but
    leaves the L2 full of dirty lines that the first kernel of the next step
    would then write back to HBM inside its timed region (~100 MB for C2's
    initial LayerNorm, which doubled its DRAM traffic).  Reading a second
    buffer of the same size afterwards forces those write-backs here, untimed,
    and leaves clean lines of an unrelated buffer.
    """

    def __init__(self, device: torch.device) -> None:
        self._write = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        self._read = torch.zeros(L2_FLUSH_BYTES // 8, dtype=torch.int64, device=device)

    def __call__(self) -> None:
        self._write.zero_()
        self._sink = self._read.sum()



def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def _peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# Committed ncu summary of each kernel role at C2 (profiles/<name>_c2.txt).
PROFILE_OF_ROLE = {
    "attention": "attention",
    "ffn_input_projection": "gemm_ffn_in_gelu",
    "residual_norm": "residual_layernorm",
}


def _profile_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary, if any."""

    path = REPO / "profiles" / f"{PROFILE_OF_ROLE.get(kernel, kernel)}_c2.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle",
        0x2: "applications_clocks_setting",
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int, period_s: float = 0.005) -> None:
        self.device_index = device_index
        self.period_s = period_s
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz: int | None = None
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._nvml = None

    def __enter__(self) -> ClockSampler:
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid_index = self.device_index
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            if visible:
                parts = [p.strip() for p in visible.split(",") if p.strip()]
                if self.device_index < len(parts) and parts[self.device_index].isdigit():
                    uuid_index = int(parts[self.device_index])
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(uuid_index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nvml = None
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self) -> None:
        pynvml = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(int(pynvml.nvmlDeviceGetClockInfo(self._handle, pynvml.NVML_CLOCK_SM)))
                mask = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(self._handle))
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period_s)

    def __exit__(self, *exc: object) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass

    def summary(self) -> dict:
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


# ---------------------------------------------------------------- CPU baseline
REFERENCE_INSTALL = REPO / "baseline" / "_ref"
# The head-sharded parity check of N >= 2 runs (groups of two ranks): small
# enough that the reference's CPU forward takes well under a second.
TP_PARITY_SPEC = dict(batch_size=2, seq_len=256, d_model=512, num_heads=8, ffn_dim=2048, num_layers=2, causal=True)
TP_PARITY_SEED = 11
PARITY_MAX_ABS = 2e-2
PARITY_REL_L2 = 1e-2


def _host_threads() -> int:
    """Use every host core for the CPU legs, whatever torchrun's
    OMP_NUM_THREADS=1 says; returns the thread count."""

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return threads


def _reference_module():  # noqa: ANN202
    """The reference's official harness (official/torch_transformer_benchmark.py)
    from its install in baseline/_ref, or None when it is not installed.  Only
    the CPU legs below use it."""

    if not (REFERENCE_INSTALL / "official" / "torch_transformer_benchmark.py").exists():
        return None
    path = str(REFERENCE_INSTALL)
    if path not in sys.path:
        # Appended: the package's own `solution` and `deployment` stay first;
        # `official` exists only in the reference install.
        sys.path.append(path)
    import importlib

    return importlib.import_module("official.torch_transformer_benchmark")


def reference_cpu_forward(spec: dict, x: torch.Tensor, steps: int, warmup: int) -> dict:
    """Time the reference's own CPU forward on ``x`` ([rows, S, D] fp32).

    ``official.BaselineTransformer`` built after ``torch.manual_seed(0)`` (the
    weights of every GPU run here), timed by the reference's own
    ``benchmark_once`` (perf_counter_ns around each forward on CPU, official
    :477-506) on all host cores.  Without the reference install the numpy
    restatement of the same forward (oracle/) is timed instead (kind "port").
    Returns the timing and the output of the forward.
    """

    threads = _host_threads()
    rows, seq = int(x.shape[0]), int(x.shape[1])
    ref = _reference_module()
    if ref is not None:
        config = ref.TransformerConfig(**{**spec, "batch_size": rows})
        saved = torch.get_rng_state()
        torch.manual_seed(WEIGHT_SEED)
        model = ref.BaselineTransformer(config).eval()
        torch.set_rng_state(saved)
        mask = torch.ones(rows, seq, dtype=torch.bool)
        with torch.inference_mode():
            output = model(x, mask)
        if warmup > 1:
            ref.benchmark_once(model, x, mask, warmup - 1, torch.device("cpu"))
        samples_ms = ref.benchmark_once(model, x, mask, max(1, steps), torch.device("cpu"))
        kind = "reference"
        what = "official.BaselineTransformer fp32 forward (the reference's PyTorch CPU path, from baseline/_ref)"
        output = output.numpy()
    else:
        from threadpoolctl import threadpool_limits

        from oracle import OfficialConfig, official_state_dict
        from oracle.reference_forward import transformer_forward
        from oracle.weights import state_to_numpy

        cfg = OfficialConfig(**{**spec, "batch_size": rows})
        state = state_to_numpy(official_state_dict(cfg, seed=WEIGHT_SEED))
        kwargs = dict(num_heads=cfg.num_heads, num_layers=cfg.num_layers, causal=cfg.causal)
        xs = x.numpy()
        with threadpool_limits(threads):
            output = transformer_forward(xs, state, **kwargs)
            for _ in range(max(0, warmup - 1)):
                transformer_forward(xs, state, **kwargs)
            samples_ms = []
            for _ in range(max(1, steps)):
                start = time.perf_counter_ns()
                transformer_forward(xs, state, **kwargs)
                samples_ms.append((time.perf_counter_ns() - start) / 1e6)
        kind = "port"
        what = "numpy fp32 restatement of the reference forward (reference install absent)"
    per_step = statistics.median(samples_ms) / 1000.0
    return {
        "value": rows * seq / per_step,
        "unit": UNIT,
        "cores": threads,
        "kind": kind,
        "sample": f"{what}: {rows} batch row(s) x {seq} tokens per sample, median of {len(samples_ms)}",
        "seconds_per_sample": per_step,
        "output": output,
    }


def _errors(got: torch.Tensor | object, ref: object) -> dict:
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = got - ref
    max_abs = float(np.abs(diff).max())
    rel = float(np.linalg.norm(diff) / max(np.linalg.norm(ref), 1e-30))
    return {"max_abs": max_abs, "rel_l2": rel, "ok": max_abs <= PARITY_MAX_ABS and rel <= PARITY_REL_L2}


def run_reference(args: argparse.Namespace) -> None:
    """The reference arm: the reference's own CPU forward on one batch row of
    the C2 workload per step (rank 0 only under torchrun)."""

    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    from workloads import WorkloadConfig, seeded_input

    x = seeded_input(WorkloadConfig(**WORKLOAD), INPUT_SEED)[:1].contiguous()
    base = reference_cpu_forward(WORKLOAD, x, steps=args.steps, warmup=min(args.warmup, 2))
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": base["value"],
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": base["seconds_per_sample"] * 1000.0,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) input, seeded default-init weights)",
        "config": {"workload": WORKLOAD_NAME, "sample": "one batch row per step", "global_batch": 1,
                   "seq_len": WORKLOAD["seq_len"], "parallelism": "cpu"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def build_model(device: torch.device, spec: dict | None = None):
    from solution.transformer import UserOptimizedTransformer, copy_model_weights
    from workloads import WorkloadConfig, seeded_state_dict

    spec = spec or WORKLOAD
    model = UserOptimizedTransformer(SimpleNamespace(**spec))
    copy_model_weights(seeded_state_dict(WorkloadConfig(**spec), seed=WEIGHT_SEED), model)
    return model.to(device).eval()


def _c4_tp(args: argparse.Namespace, batch: int, world: int) -> int:
    """Tensor-parallel group size of the head-sharded C4 run: --tp, else the
    smallest head sharding (2) that, with data-parallel replicas over the
    batch rows, covers all ranks (B=4: tp2 on 2, dp2 x tp2 on 4, dp4 x tp2 on 8
    GPUs; measured fastest on 8 GPUs, where tp8 all-reduces 4x the bytes)."""

    if args.tp:
        return args.tp
    tp = max(2, world // batch)
    return tp if world % tp == 0 else world


def _workload_input(name: str, args: argparse.Namespace, spec: dict, seed: int, rank: int, world: int):
    """This rank's input rows and the parallel mode of the workload."""

    from solution.runtimes.sharded import batch_shard_bounds
    from workloads import WorkloadConfig, seeded_input, seeded_row

    cfg = WorkloadConfig(**spec)
    if name == "c4" and world > 1:
        # Head-sharded tensor parallel over groups of --tp ranks; the
        # world // tp replicas split the batch rows between them.
        tp = _c4_tp(args, cfg.batch_size, world)
        start, stop = batch_shard_bounds(cfg.batch_size, rank // tp, world // tp)
        x = seeded_input(cfg, seed)[start:stop].contiguous()
        return x, "heads", "strong", cfg.batch_size * cfg.seq_len
    if name == "c5":
        # Batch-sharded capacity run: the 32 rows (seed 4 + row) split over ranks.
        start, stop = batch_shard_bounds(cfg.batch_size, rank, world)
        rows = [seeded_row(cfg, seed, r) for r in range(start, stop)]
        x = torch.cat(rows, dim=0)
        return x, "batch", "strong", cfg.batch_size * cfg.seq_len
    # c2 / c3: every rank runs its own full batch (rank r: seed + r).
    return seeded_input(cfg, seed + rank), "batch", "weak", world * cfg.batch_size * cfg.seq_len


GEMM_VARIANT_NAMES = {0: "1SM", 1: "PAIR", 2: "WARP"}
ATTENTION_VARIANT_NAMES = {0: "PAIRED", 1: "SINGLE", 2: "QUAD", 3: "PERSISTENT", 4: "DUO", 5: "PINGPONG"}


def _program(model, runner) -> dict:  # noqa: ANN001
    """The program that ran: its config id, where the config came from
    (a deployed entry for this environment and shape, or the default), the
    runtime and the kernel variant of each launch."""

    config = model.active_config
    schedule = config.schedule

    def gemm(launch) -> str:  # noqa: ANN001
        return GEMM_VARIANT_NAMES[launch.kernel_variant if launch is not None else 1]

    program = {
        "config_id": config.config_id,
        "source": model.active_config_source,
        "runtime": schedule.runtime.value,
        "attention": config.program.attention.value,
        "attention_variant": (
            ATTENTION_VARIANT_NAMES[schedule.attention_launch.kernel_variant]
            if schedule.attention_launch is not None
            else None
        ),
        "gemm": {
            "qkv": gemm(schedule.qkv_launch),
            "out_proj": gemm(schedule.attention_output_projection_launch),
            "ffn_in": gemm(schedule.ffn_input_launch),
            "ffn_out": gemm(schedule.ffn_launch),
        },
    }
    if runner is not model:
        # The head-sharded runner launches its own fixed program.
        program = {"runner": type(runner).__name__, "reduction": runner.reduction,
                   "attention_variant": "QUAD", "gemm": "PAIR", "runtime": "eager"}
    return program


class _Context(SimpleNamespace):
    """What every workload of one bench run shares: flags, ranks, device."""


def measure_workload(ctx: _Context, name: str, steps: int, warmup: int, full: bool) -> dict:
    """Time ``steps`` forwards of one BASELINE workload on every rank.

    Every rank takes the same collective steps in the same order.  With
    ``full`` (the headline workload) it also runs the per-kernel event pass
    for the roofline and the end-to-end host pipeline; the other workloads
    run a one-step kernel pass (single-GPU program only) for their attention
    time.  Returns rank-local results and the max-over-ranks times.
    """

    from solution.runtimes.sharded import TensorParallelTransformer
    from solution.transformer import KernelEventRecorder
    from workloads import WorkloadConfig

    args, dist, rank, world, device = ctx.args, ctx.dist, ctx.rank, ctx.world, ctx.device
    spec, seed, title = WORKLOADS[name]
    cfg = WorkloadConfig(**spec)
    model = build_model(device, spec)
    x_cpu, parallel, scaling, total_tokens = _workload_input(name, args, spec, seed, rank, world)
    tp = 1
    if parallel == "heads":
        from solution.runtimes.sharded import tensor_parallel_groups

        tp = _c4_tp(args, cfg.batch_size, world)
        group, _, _ = tensor_parallel_groups(tp)
        partials = torch.bfloat16 if args.tp_partials == "bf16" else torch.float32
        reduction = args.tp_reduction if args.tp_reduction != "auto" else ("peer" if tp <= 4 else "nccl")
        # peer: the whole partials of every peer for groups of two, the
        # reduce-scatter + gather form for larger groups; peer-full and
        # peer-scatter force one of them.
        scatter = {"peer-full": False, "peer-scatter": True}.get(reduction)
        # The error word is read once after all steps (device_error below),
        # not after every step, so the host keeps running ahead of the GPU.
        runner = TensorParallelTransformer(
            model, group=group, partial_dtype=partials, reduction="nccl" if reduction == "nccl" else "peer",
            check_peer_errors=False, peer_scatter=scatter,
        )
    else:
        reduction = None
        runner = model
    x_host = x_cpu.pin_memory() if full else None
    x_dev = (x_host if full else x_cpu).to(device)
    del x_cpu
    big_input = x_dev.numel() * x_dev.element_size() > 2 * L2_FLUSH_BYTES
    flush = None if big_input else L2Flush(device)
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)

    def barrier() -> None:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    first_row = None
    with torch.inference_mode():
        for i in range(warmup):
            y = runner(x_dev)
            if i == 0 and full and rank == 0 and world == 1:
                first_row = y[:1].float().cpu()
            del y
        torch.cuda.synchronize()

        # Timed steps: nothing but the forward between the step's two events,
        # so consecutive kernels keep their programmatic launch overlap.
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier()
        with ClockSampler(ctx.local_rank) as clocks:
            for i in range(steps):
                if flush is not None:
                    flush()
                starts[i].record()
                runner(x_dev)
                ends[i].record()
            barrier()
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        # Peak device memory of the forward itself (the host pipeline below
        # adds its own input slots).
        peak_gb = torch.cuda.max_memory_allocated(device) / 2**30

        # Per-kernel times for the kernel table and the roofline: the same
        # program again with CUDA events around every launch (these events sit
        # between kernels, so this pass is not the step time).  A graph
        # runtime replays its launches where the events cannot sit, so this
        # pass runs the same program under the eager runtime.
        kernel_ms: dict[str, list[float]] = {}
        event_floor_us = None
        kernel_steps = steps if full else 1
        if runner is model:
            from dataclasses import replace as _replace

            from solution.config import RuntimeBackend

            graph_config = None
            if model.active_config.schedule.runtime in (
                RuntimeBackend.CUDA_GRAPH,
                RuntimeBackend.BATCH_TILED_CUDA_GRAPH,
            ):
                graph_config = model.active_config
                graph_source = model.active_config_source
                model.configure_execution(
                    config=_replace(
                        graph_config,
                        schedule=_replace(graph_config.schedule, runtime=RuntimeBackend.EAGER, batch_tile_size=None),
                    )
                )
            recorder = KernelEventRecorder()
            model.kernel_events = recorder
            for _ in range(kernel_steps):
                if flush is not None:
                    flush()
                runner(x_dev)
            torch.cuda.synchronize()
            model.kernel_events = None
            kernel_ms = recorder.durations_ms()
            if graph_config is not None:
                model.configure_execution(config=graph_config)
                model.active_config_source = graph_source
            # The floor of that method: a one-element fill bracketed by the
            # same two events after the same flush (event processing and the
            # launch gap it adds to every kernel's figure).
            tiny = torch.empty(1, device=device)
            floor_ms = []
            for _ in range(max(5, kernel_steps)):
                if flush is not None:
                    flush()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                tiny.zero_()
                e1.record()
                floor_ms.append((e0, e1))
            torch.cuda.synchronize()
            floor_ms = sorted(a.elapsed_time(b) for a, b in floor_ms)
            event_floor_us = 1000.0 * floor_ms[len(floor_ms) // 2]

        e2e_ms = 0.0
        out_host = None
        if full:
            # End to end through the public host-batch API (HostPipeline) from
            # pinned host memory: every step copies its input H2D, runs the
            # forward and copies the whole output D2H; the three run on
            # separate streams, so step i's forward overlaps step i+1's
            # copy-in and step i-1's copy-out.  Timed by CUDA events from
            # before the first copy-in to after the last copy-out.
            from solution.runtimes.host_pipeline import HostPipeline

            pipe = HostPipeline(runner, device, depth=3)
            outs_host = [torch.empty(x_host.shape, dtype=x_host.dtype).pin_memory() for _ in range(2)]
            for i in range(3):
                pipe.submit(x_host, outs_host[i % 2])
            pipe.synchronize()
            barrier()
            e2e_start = torch.cuda.Event(enable_timing=True)
            e2e_end = torch.cuda.Event(enable_timing=True)
            e2e_start.record(pipe.copy_in)
            for i in range(steps):
                pipe.submit(x_host, outs_host[i % 2])
            e2e_end.record(pipe.copy_out)
            pipe.synchronize()
            barrier()
            e2e_ms = e2e_start.elapsed_time(e2e_end) / steps
            out_host = outs_host[0]
            # The host link alone, all ranks at once: the step's input copied
            # H2D, then its output D2H, then both directions together (on two
            # streams), each timed by CUDA events -- the rates that bound e2e.
            # "both": the two directions on two streams with no dependency
            # between them, as the pipeline runs them.
            link = torch.empty_like(x_dev)
            up = torch.cuda.Stream(device)
            down = torch.cuda.Stream(device)
            link_ms = {}
            reps = 5
            for name in ("h2d", "d2h", "both"):
                barrier()
                t0 = torch.cuda.Event(enable_timing=True)
                t1 = torch.cuda.Event(enable_timing=True)
                t0.record()
                up.wait_event(t0)
                down.wait_event(t0)
                for _ in range(reps):
                    if name in ("h2d", "both"):
                        with torch.cuda.stream(up):
                            link.copy_(x_host, non_blocking=True)
                    if name in ("d2h", "both"):
                        with torch.cuda.stream(down):
                            out_host.copy_(x_dev, non_blocking=True)
                cur = torch.cuda.current_stream(device)
                cur.wait_stream(up)
                cur.wait_stream(down)
                t1.record()
                torch.cuda.synchronize(device)
                link_ms[name] = t0.elapsed_time(t1) / reps
            del link

    total_ms = sum(step_ms)
    link_vals = [link_ms.get(k, 0.0) for k in ("h2d", "d2h", "both")] if full else [0.0, 0.0, 0.0]
    stats = torch.tensor([total_ms, e2e_ms, peak_gb, *link_vals], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    total_ms_max, e2e_ms_max, peak_gb_max, h2d_ms, d2h_ms, both_ms = stats.tolist()
    ms_per_step = total_ms_max / steps

    b_loc = x_dev.shape[0]
    s, d, f, layers = cfg.seq_len, cfg.d_model, cfg.ffn_dim, cfg.num_layers
    m = b_loc * s
    heads_frac = 1.0 / tp
    # Algorithmic work of one step per kernel role (the streamed runtime
    # splits it over several launches per layer, so work and time are both
    # taken per step): FLOPs for the tensor-core kernels (causal attention
    # counted as 2BS^2D like the reference), HBM bytes for the norms.
    flops_per_step = {
        "attention": layers * 2.0 * b_loc * s * s * d * heads_frac,
        "qkv_projection": layers * 2.0 * m * 3 * d * d * heads_frac,
        "attention_output_projection": layers * 2.0 * m * d * d * heads_frac,
        "ffn_input_projection": layers * 2.0 * m * f * d * heads_frac,
        "ffn_output_projection": layers * 2.0 * m * d * f * heads_frac,
    }
    # Residual LN: read r (fp32) + u (bf16), write r (fp32) + n (bf16) = 12 B per
    # element; the last one writes no residual and the output in the input's
    # dtype: 4 + 2 + out bytes.  Initial LN: read x, write bf16 n.
    io_bytes = float(x_dev.element_size())
    bytes_per_step = {
        "residual_norm": ((2 * layers - 1) * 12.0 + 6.0 + io_bytes) * m * d,
        "initial_norm": (io_bytes + 2.0) * m * d,
    }
    per_role = {role: sum(v) / kernel_steps for role, v in kernel_ms.items()}
    launches = {role: len(v) // kernel_steps for role, v in kernel_ms.items()}
    peaks, peak_source = _peaks()
    roofline = None
    if per_role:
        dominant = max(per_role, key=per_role.get)
        role_s = per_role[dominant] / 1000.0
        n_launch = max(1, launches[dominant])
        if dominant in flops_per_step:
            achieved = flops_per_step[dominant] / role_s / 1e12
            # Kernels timed inside a step of a few milliseconds: the burst
            # GEMM peak (the sustained figure is for seconds-long loops).
            peak = float(peaks["bf16_tflops"])
            roofline = {"bound": "tensor", "unit": "TFLOP/s", "kernel": dominant,
                        "algorithmic_per_launch": flops_per_step[dominant] / n_launch}
            peak_name = "bf16_tflops (burst)"
        else:
            achieved = bytes_per_step[dominant] / role_s / 1e9
            peak = float(peaks["hbm_gbs"])
            roofline = {"bound": "hbm", "unit": "GB/s", "kernel": dominant,
                        "algorithmic_per_launch": bytes_per_step[dominant] / n_launch}
            peak_name = "hbm_gbs"
        roofline.update(
            achieved=achieved,
            peak=peak,
            peak_source=f"{peak_source} ({peak_name})",
            frac=achieved / peak,
            traffic=_profile_traffic(dominant) if name == "c2" else None,
            avg_launch_ms=per_role[dominant] / n_launch,
        )
    attention_s = per_role.get("attention", 0.0) / 1000.0
    attention_tflops = flops_per_step["attention"] / attention_s / 1e12 if attention_s else None
    model_flops = (total_tokens / cfg.seq_len) * layers * (2.0 * s * s * d + 8.0 * s * d * d + 4.0 * s * d * f)
    parallelism = (
        (f"dp{world // tp} x " if tp < world else "")
        + (
            f"tp{tp} (head-sharded, NCCL all-reduce of {args.tp_partials} partials after out-proj and FFN-down)"
            if reduction == "nccl"
            else (
                f"tp{tp} (head-sharded, each rank sums the group's bf16 partials for its slice of the rows over "
                "NVLink peer memory inside the residual LayerNorm and writes the normalised slice into every "
                "rank's buffer, after out-proj and FFN-down)"
                if getattr(getattr(runner, "_peer", None), "scatter", False)
                else f"tp{tp} (head-sharded, bf16 partials summed over NVLink peer memory inside the residual "
                "LayerNorm after out-proj and FFN-down)"
            )
        )
        if parallel == "heads"
        else f"dp{world} (batch-sharded, no collective)"
    )
    result = {
        "workload": title,
        "value": total_tokens * steps / (total_ms_max / 1000.0),
        "unit": UNIT,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms_per_step,
        "p50_latency_ms": statistics.median(step_ms),
        "scaling": scaling,
        "global_batch": cfg.batch_size * (world if scaling == "weak" else 1),
        "seq_len": cfg.seq_len,
        "parallelism": parallelism,
        "l2": "inputs larger than L2" if big_input else L2_FLUSH_NOTE,
        "program": _program(model, runner),
        "attention_tflops": attention_tflops,
        "attention_frac_of_burst": attention_tflops / float(peaks["bf16_tflops"]) if attention_tflops else None,
        "model_tflops": model_flops / (ms_per_step / 1000.0) / 1e12,
        "peak_memory_gb_per_gpu": peak_gb_max,
        "clocks": clocks.summary(),
        # rank-local extras for the headline line
        "_kernels": {role: {"ms_per_step": per_role[role], "launches_per_step": launches[role]}
                     for role in sorted(per_role)},
        "_event_floor_us": event_floor_us,
        "_roofline": roofline,
        "_launches": int(sum(len(v) for v in kernel_ms.values())),
        "_e2e_ms": e2e_ms_max,
        "_total_tokens": total_tokens,
        "_first_row": first_row,
        "_host_link": (
            {
                "bytes_per_rank_each_way": int(x_host.numel() * x_host.element_size()),
                "ranks_copying_at_once": world,
                "h2d_gbs_per_rank": x_host.numel() * x_host.element_size() / (h2d_ms / 1000.0) / 1e9,
                "d2h_gbs_per_rank": x_host.numel() * x_host.element_size() / (d2h_ms / 1000.0) / 1e9,
                "both_directions_ms": both_ms,
                "both_directions_gbs_per_rank": 2 * x_host.numel() * x_host.element_size() / (both_ms / 1000.0) / 1e9,
                "h2d_then_d2h_ms": h2d_ms + d2h_ms,
                "timing": "CUDA events, slowest rank, 5 copies each, pinned host memory; 'both' runs "
                          "the two directions on two independent streams",
            }
            if full and h2d_ms > 0
            else None
        ),
        "_h2d": int(x_host.numel() * x_host.element_size()) if x_host is not None else 0,
        "_d2h": int(out_host.numel() * out_host.element_size()) if out_host is not None else 0,
    }
    if hasattr(runner, "close"):
        runner.close()
    del runner, model, x_dev, x_host, flush
    torch.cuda.empty_cache()
    barrier()
    return result


def tensor_parallel_parity(ctx: _Context) -> dict:
    """Head-sharded forward (groups of two ranks, NCCL and peer reductions)
    of a small workload against the reference's CPU forward on the same
    seeded input and weights.  Every rank runs its group's forward; rank 0
    compares its result.  Returns rank 0's report (empty elsewhere)."""

    from solution.runtimes.sharded import TensorParallelTransformer, tensor_parallel_groups
    from workloads import WorkloadConfig, seeded_input

    dist, rank, device = ctx.dist, ctx.rank, ctx.device
    cfg = WorkloadConfig(**TP_PARITY_SPEC)
    group, _, _ = tensor_parallel_groups(2)
    model = build_model(device, TP_PARITY_SPEC)
    x = seeded_input(cfg, TP_PARITY_SEED)
    outputs = {}
    for reduction in ("nccl", "peer"):
        runner = TensorParallelTransformer(model, group=group, partial_dtype=torch.bfloat16, reduction=reduction)
        with torch.inference_mode():
            outputs[reduction] = runner(x.to(device)).float().cpu()
        torch.cuda.synchronize()
        runner.close()
    dist.barrier()
    del model
    torch.cuda.empty_cache()
    if rank != 0:
        return {}
    reference = reference_cpu_forward(TP_PARITY_SPEC, x, steps=1, warmup=1)
    report = {
        "workload": "B2 S256 D512 H8(Dh64) F2048 L2 causal, x seed 11, fp32 I/O",
        "group": "tp2 (ranks 0-1)",
        "against": reference["kind"],
        "tolerance": {"max_abs": PARITY_MAX_ABS, "rel_l2": PARITY_REL_L2},
    }
    for reduction, y in outputs.items():
        report[reduction] = _errors(y.numpy(), reference["output"])
    return report


def run_gpu(args: argparse.Namespace) -> None:
    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local_rank = _env_int("LOCAL_RANK", 0)
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist_mod

        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        dist = dist_mod

    from solution import _native

    _native.device_check()
    ctx = _Context(args=args, dist=dist, rank=rank, world=world, local_rank=local_rank, device=device)
    warmup = max(3, args.warmup)
    main = measure_workload(ctx, args.workload, args.steps, warmup, full=True)
    extras: dict[str, dict] = {}
    if args.workload == "c2" and args.extras != "none":
        for name in (n.strip() for n in args.extras.split(",")):
            if not name:
                continue
            if name not in WORKLOADS:
                raise SystemExit(f"--extras: unknown workload {name!r} (choose from {sorted(WORKLOADS)} or 'none')")
            steps = {"c3": args.steps, "c4": min(args.steps, 10), "c5": min(args.steps, 3)}.get(name, args.steps)
            extras[name] = measure_workload(ctx, name, steps, 3, full=False)
    tp_parity = tensor_parallel_parity(ctx) if world >= 2 and not args.skip_tp_parity else None
    device_error = _native.device_error(clear=True)

    if rank == 0:
        spec = WORKLOADS[args.workload][0]
        launches_per_step = 1 + 7 * spec["num_layers"]
        line = {
            "metric": METRIC,
            "value": main["value"],
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": warmup,
            "ms_per_step": main["ms_per_step"],
            "p50_latency_ms": main["p50_latency_ms"],
            "higher_is_better": True,
            "scaling": main["scaling"],
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: x ~ N(0,1) from the BASELINE seeds (CPU generator), reference default-init weights seed 0",
            "config": {
                "workload": main["workload"],
                "global_batch": main["global_batch"],
                "seq_len": main["seq_len"],
                "parallelism": main["parallelism"],
                "io_dtype": "float32 in/out, bf16 GEMM/attention operands, fp32 accumulation and residual",
                "l2": main["l2"],
                "runtime": main["program"].get("runtime"),
                "program": main["program"],
            },
            "attention_tflops": main["attention_tflops"],
            "attention_frac_of_burst": main["attention_frac_of_burst"],
            "model_tflops": main["model_tflops"],
            "peak_memory_gb_per_gpu": main["peak_memory_gb_per_gpu"],
            "kernels": main["_kernels"],
            "kernel_event_floor_us": main["_event_floor_us"],
            "roofline": main["_roofline"],
            "e2e": {
                "value": main["_total_tokens"] / (main["_e2e_ms"] / 1000.0),
                "unit": UNIT,
                "h2d_bytes_per_step": main["_h2d"],
                "d2h_bytes_per_step": main["_d2h"],
                "ms_per_step": main["_e2e_ms"],
                "host_link": main["_host_link"],
            },
            "gpu_launches": main["_launches"] or launches_per_step * args.steps,
            "clocks": main["clocks"],
            "device_error": device_error,
        }
        if extras:
            line["workloads"] = {
                name: {k: v for k, v in result.items() if not k.startswith("_")} for name, result in extras.items()
            }
        if tp_parity is not None:
            line["tp_parity"] = tp_parity
        if world == 1 and args.workload == "c2" and not args.skip_cpu_baseline:
            # The reference's CPU forward on row 0 of the same C2 batch, timed
            # on this host's cores (>= 3 samples); its output is also the
            # parity check of this run's GPU output row.
            from workloads import WorkloadConfig, seeded_input

            x0 = seeded_input(WorkloadConfig(**WORKLOAD), INPUT_SEED)[:1].contiguous()
            base = reference_cpu_forward(WORKLOAD, x0, steps=3, warmup=1)
            line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
            if main["_first_row"] is not None:
                line["reference_parity"] = {
                    "rows": "batch row 0 of the C2 input",
                    "against": base["kind"],
                    **_errors(main["_first_row"].numpy(), base["output"]),
                }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_kernel(args: argparse.Namespace) -> None:
    """Time one libb200tx kernel on its C2 operands (CUDA events, L2 flushed)."""

    from solution import _native

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _native.device_check()
    g = torch.Generator(device=device).manual_seed(0)
    b, s, d, h, f = (WORKLOAD[k] for k in ("batch_size", "seq_len", "d_model", "num_heads", "ffn_dim"))
    if args.shape:
        b, s, h = (int(v) for v in args.shape.split(","))
        d = h * 64
        f = 4 * d
    m = b * s

    def randn(*shape, scale=1.0, dtype=torch.bfloat16):
        return (torch.randn(*shape, device=device, generator=g) * scale).to(dtype)

    gemm = {
        "qkv": (d, 3 * d, False),
        "out_proj": (d, d, False),
        "ffn_in": (d, f, True),
        "ffn_out": (f, d, False),
    }
    if args.kernel.startswith("attention"):
        qkv = randn(b, s, 3 * d)
        out = torch.empty(b, s, d, device=device, dtype=torch.bfloat16)
        variant = {
            "attention": _native.ATTN_QUAD,
            "attention_paired": _native.ATTN_PAIRED,
            "attention_single": _native.ATTN_SINGLE,
            "attention_persistent": _native.ATTN_PERSISTENT,
            "attention_duo": _native.ATTN_DUO,
            "attention_pingpong": _native.ATTN_PINGPONG,
        }[args.kernel]
        launch = lambda: _native.attention(qkv, out, b, s, h, 64, 0.125, True, variant)  # noqa: E731
        work, unit, bound = 2.0 * b * s * s * d, "TFLOP/s", "tensor"
    elif args.kernel.removesuffix("_pair") in gemm:
        k, n, gelu = gemm[args.kernel.removesuffix("_pair")]
        variant = _native.GEMM_PAIR if args.kernel.endswith("_pair") else _native.GEMM_1SM
        a = randn(m, k)
        w = randn(n, k, scale=k**-0.5)
        bias = randn(n, dtype=torch.float32)
        out = torch.empty(m, n, device=device, dtype=torch.bfloat16)
        epi = _native.EPI_BIAS_GELU if gelu else _native.EPI_BIAS
        launch = lambda: _native.linear(a, w, bias, out, epi, variant)  # noqa: E731
        work, unit, bound = 2.0 * m * n * k, "TFLOP/s", "tensor"
    elif args.kernel == "initial_norm":
        x = randn(m, d, dtype=torch.float32)
        normed = torch.empty(m, d, device=device, dtype=torch.bfloat16)
        gamma = torch.ones(d, device=device)
        beta = torch.zeros(d, device=device)
        launch = lambda: _native.residual_layer_norm(x, None, None, normed, gamma, beta, 1e-5)  # noqa: E731
        work, unit, bound = 6.0 * m * d, "GB/s", "hbm"
    elif args.kernel == "residual_norm":
        resid = randn(m, d, dtype=torch.float32)
        upd = randn(m, d)
        normed = torch.empty(m, d, device=device, dtype=torch.bfloat16)
        gamma = torch.ones(d, device=device)
        beta = torch.zeros(d, device=device)
        launch = lambda: _native.residual_layer_norm(resid, upd, resid, normed, gamma, beta, 1e-5)  # noqa: E731
        work, unit, bound = 12.0 * m * d, "GB/s", "hbm"
    else:
        raise SystemExit(f"unknown kernel {args.kernel}")
    flush = L2Flush(device)
    for _ in range(max(3, args.warmup)):
        launch()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush()
        starts[i].record()
        launch()
        ends[i].record()
    torch.cuda.synchronize()
    if _native.device_error() != 0:
        raise SystemExit("a kernel wait timed out")
    ms = statistics.median(s.elapsed_time(e) for s, e in zip(starts, ends))
    peaks, source = _peaks()
    if unit == "TFLOP/s":
        achieved = work / (ms / 1000.0) / 1e12
        peak = float(peaks["bf16_tflops"])
    else:
        achieved = work / (ms / 1000.0) / 1e9
        peak = float(peaks["hbm_gbs"])
    print(json.dumps({
        "kernel": args.kernel,
        "workload": WORKLOAD_NAME if not args.shape else f"B{b} S{s} H{h} D{d} F{f}",
        "ms": ms, "achieved": achieved, "unit": unit,
        "bound": bound, "peak": peak, "peak_source": f"{source} burst", "frac": achieved / peak,
        "steps": args.steps,
    }), flush=True)


def official_schedules(cfg, eager: bool = False) -> list[tuple[str, object]]:  # noqa: ANN001
    """The named schedules the official-shapes table times for one shape:
    ``graph`` (the default program under the CUDA-graph runtime),
    ``graph_warp_gemm`` (every projection on the small-problem GEMM) and, for
    d_model 32/64/128, ``graph_fused_{linear,mlp}[_warp_gemm]`` (the fused
    block boundaries, optionally with the remaining projections on the
    small-problem GEMM), and, where it is built, ``sequence_resident`` (the
    whole forward in one kernel).  ``eager`` runs the other programs under the
    eager runtime (one launch per kernel, for ncu launch lists)."""

    import dataclasses

    from solution.config import (
        ConfigSpec,
        RuntimeBackend,
        Sm100GemmParams,
        default_attention,
        default_program,
        default_schedule,
    )

    runtime = RuntimeBackend.EAGER if eager else RuntimeBackend.CUDA_GRAPH
    attention = default_attention(cfg.d_model // cfg.num_heads)
    warp = Sm100GemmParams(64, 64, 64, 1)
    graph = default_schedule(runtime, attention=attention)
    out = [
        ("graph", ConfigSpec(program=default_program(attention=attention), schedule=graph)),
        ("graph_warp_gemm", ConfigSpec(
            program=default_program(attention=attention),
            schedule=dataclasses.replace(
                graph, qkv_launch=warp, attention_output_projection_launch=warp, ffn_input_launch=warp,
                ffn_launch=warp,
            ),
        )),
    ]
    if cfg.d_model in (32, 64, 128):
        for fusion in ("linear", "mlp") if cfg.ffn_dim % 16 == 0 else ("linear",):
            fused = default_schedule(runtime, attention=attention, fused_boundary=fusion)
            program = default_program(attention=attention, fused_boundary=fusion)
            out.append((f"graph_fused_{fusion}", ConfigSpec(program=program, schedule=fused)))
            rest = {"qkv_launch": warp, **({"ffn_input_launch": warp} if fusion == "linear" else {})}
            out.append((f"graph_fused_{fusion}_warp_gemm",
                        ConfigSpec(program=program, schedule=dataclasses.replace(fused, **rest))))
    from solution.runtimes.sequence_resident import sequence_resident_supported

    if not eager and sequence_resident_supported(
        d_model=cfg.d_model, ffn_dim=cfg.ffn_dim, num_heads=cfg.num_heads, seq_len=cfg.seq_len,
        num_layers=cfg.num_layers, causal=bool(cfg.causal),
    ) is None:
        # The whole forward in one kernel (csrc/seq_forward_kernels.cuh).
        out.append(("sequence_resident", ConfigSpec(
            program=default_program(attention=attention),
            schedule=default_schedule(RuntimeBackend.SEQUENCE_RESIDENT, attention=attention),
        )))
    return out


def run_official(args: argparse.Namespace) -> None:
    """The reference's headline table on one B200: its official shapes.

    The reference publishes, per official shape, the median forward latency
    of its deployed program and of the official PyTorch baseline on one
    RTX 4080 (fp32 I/O; workloads.REFERENCE_PUBLISHED_MS).  This mode runs the
    same shapes (fp32 input from seed 0, weights from seed 0) through
    ``UserOptimizedTransformer`` with the config it resolves by itself (the
    deployed entry for this device and shape, else the eager default), with
    the CUDA-graph schedule, with the CUDA-graph schedule on the small-problem
    GEMM variant and, for d_model <= 128, with the fused block boundaries, each
    forward bracketed by CUDA events after an L2
    flush, and reports the median of each schedule beside the published
    numbers.  official_14 (B32 S100000, the streamed capacity shape) runs its
    default streamed config with at most 2 timed forwards.
    """

    from solution import _native
    from workloads import OFFICIAL_SHAPES, REFERENCE_PUBLISHED_MS, seeded_input, seeded_row

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _native.device_check()
    flush = L2Flush(device)
    cases = args.cases.split(",") if args.cases else sorted(OFFICIAL_SHAPES)

    def median_ms(model, x, warmup: int, steps: int) -> float:  # noqa: ANN001
        with torch.inference_mode():
            for _ in range(warmup):
                model(x)
            torch.cuda.synchronize()
            times = []
            for _ in range(steps):
                flush()
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record()
                model(x)
                end.record()
                torch.cuda.synchronize()
                times.append(start.elapsed_time(end))
        return statistics.median(times)

    shapes: dict[str, dict] = {}
    with ClockSampler(0) as clocks:
        for case in cases:
            cfg = OFFICIAL_SHAPES[case]
            streamed = case == "official_14"
            if streamed:
                x_cpu = torch.cat([seeded_row(cfg, 0, r) for r in range(cfg.batch_size)])
            else:
                x_cpu = seeded_input(cfg, 0)
            x = x_cpu.to(device)
            del x_cpu
            model = build_model(device, cfg.as_dict())
            warmup, steps = (1, min(2, args.steps)) if streamed else (max(3, args.warmup), args.steps)
            row: dict = {"B": cfg.batch_size, "S": cfg.seq_len, "D": cfg.d_model, "H": cfg.num_heads,
                         "F": cfg.ffn_dim, "L": cfg.num_layers}
            # The config the model resolves by itself: its deployed entry for this
            # device and shape, else the default (eager) program.
            if args.schedule in (None, "default"):
                row["default_ms"] = median_ms(model, x, warmup, steps)
                row["default_runtime"] = model.active_config.schedule.runtime.value
            if not streamed:
                for name, config in official_schedules(cfg, args.eager_runtime):
                    if args.schedule not in (None, name):
                        continue
                    model.configure_execution(config=config)
                    row[f"{name}_ms"] = median_ms(model, x, warmup, steps)
            row["attention"] = model.active_config.program.attention.value
            timed = [v for k, v in row.items() if k.endswith("_ms")]
            if not timed:
                raise SystemExit(f"--schedule {args.schedule!r} is not timed for {case}")
            best = min(timed)
            ref_deployed, ref_baseline = REFERENCE_PUBLISHED_MS[case]
            row.update(
                best_ms=best,
                tokens_per_s=cfg.tokens / (best / 1000.0),
                ref_rtx4080_deployed_ms=ref_deployed,
                ref_rtx4080_pytorch_ms=ref_baseline,
                speedup_vs_ref_deployed=ref_deployed / best,
            )
            if ref_baseline is not None:
                row["speedup_vs_ref_pytorch"] = ref_baseline / best
            shapes[case] = row
            del model, x
            torch.cuda.empty_cache()
    if _native.device_error() != 0:
        raise SystemExit("a kernel wait timed out")

    def geomean(values: list[float]) -> float | None:
        return math.exp(sum(math.log(v) for v in values) / len(values)) if values else None

    core = [c for c in shapes if c != "official_14"]
    print(json.dumps({
        "metric": "official shapes: fwd median latency per shape",
        "unit": "ms",
        "higher_is_better": False,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "dtype": "bf16",
        "data": "synthetic (seeded x ~ N(0,1), seeded default-init weights)",
        "config": {"workload": "reference official shapes (official/test_shapes.json)", "io": "float32",
                   "l2": "flushed before every timed forward"},
        "reference_platform": "RTX 4080, published (result/20260831T083857.848038Z/final_performance.md)",
        "geomean_speedup_vs_ref_deployed_01_13": geomean([shapes[c]["speedup_vs_ref_deployed"] for c in core]),
        "geomean_speedup_vs_ref_pytorch_01_13": geomean([shapes[c]["speedup_vs_ref_pytorch"] for c in core]),
        "shapes": shapes,
        "clocks": clocks.summary(),
    }), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("native", "reference"), default="native")
    parser.add_argument("--skip-cpu-baseline", action="store_true")
    parser.add_argument("--extras", default="c3,c4,c5",
                        help="with the c2 headline: the other BASELINE configs measured after it and reported "
                             "under 'workloads' on the same line ('none' to skip)")
    parser.add_argument("--skip-tp-parity", action="store_true",
                        help="N >= 2: skip the head-sharded parity check against the reference's CPU forward")
    parser.add_argument("--workload", choices=[*sorted(WORKLOADS), "official"], default="c2",
                        help="BASELINE config to run (c2 is the bench line the driver records), "
                             "or 'official' for the reference's official-shapes table")
    parser.add_argument("--cases", default=None,
                        help="--workload official: comma-separated case ids (default: all 14)")
    parser.add_argument("--schedule", default=None,
                        help="--workload official: time only this schedule (default, graph, graph_warp_gemm, "
                             "graph_fused_linear, graph_fused_mlp, ..._warp_gemm, sequence_resident)")
    parser.add_argument("--eager-runtime", action="store_true",
                        help="--workload official: run the named schedules under the eager runtime "
                             "(one launch per kernel, for ncu launch lists)")
    parser.add_argument("--tp", type=int, default=0,
                        help="c4 under torchrun: tensor-parallel group size (default: max(2, N / B))")
    parser.add_argument("--tp-reduction", choices=("auto", "nccl", "peer", "peer-full", "peer-scatter"), default="auto",
                        help="c4: NCCL all-reduce, or the peer-memory reduction fused into the "
                             "LayerNorm: peer (whole partials for groups of 2, reduce-scatter + gather for "
                             "larger groups), peer-full / peer-scatter (forced); auto: peer for groups of up "
                             "to 4 (measured ahead of NCCL there), NCCL for 8")
    parser.add_argument("--tp-partials", choices=("fp32", "bf16"), default="bf16",
                        help="dtype of the partial sums all-reduced by the head-sharded runtime")
    parser.add_argument("--shape", default=None, help="B,S,H override for --kernel (head_dim 64, F=4D)")
    parser.add_argument(
        "--kernel",
        choices=(
            "attention",
            "attention_paired",
            "attention_single",
            "attention_persistent",
            "attention_duo",
            "attention_pingpong",
            "qkv",
            "out_proj",
            "ffn_in",
            "ffn_out",
            "qkv_pair",
            "out_proj_pair",
            "ffn_in_pair",
            "ffn_out_pair",
            "residual_norm",
            "initial_norm",
        ),
        default=None,
    )
    args = parser.parse_args()
    if args.steps <= 0:
        raise SystemExit("--steps must be positive")
    if args.impl == "reference":
        run_reference(args)
        return
    if args.kernel is not None:
        run_kernel(args)
        return
    if args.workload == "official":
        run_official(args)
        return
    run_gpu(args)


if __name__ == "__main__":
    main()
