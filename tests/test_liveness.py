"""Host-side failure detection of the multi-process runtimes
(solution/runtimes/liveness.py), without a GPU.

Failures are made on the host only: a rank that raises inside its step, a
rank that exits without a word, and a collective whose peer is gone.  The
in-process tests drive ``StepLiveness`` over a ``HashStore`` with threads as
ranks; the multi-process tests spawn gloo ranks (world size 2) whose store
is the process group's own.
"""

from __future__ import annotations

import datetime
import os
import socket
import tempfile
import threading
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from solution.runtimes.liveness import RankFailure, StepLiveness, abort_process_group


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------- in-process


def test_all_ranks_pass_each_step_boundary() -> None:
    store = dist.HashStore()
    world, steps = 3, 5
    seen: list[list[int]] = [[] for _ in range(world)]

    def rank_loop(r: int) -> None:
        live = StepLiveness(store, r, world, timeout_s=5.0)
        for _ in range(steps):
            seen[r].append(live.enter())

    threads = [threading.Thread(target=rank_loop, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=30)
    assert seen == [list(range(steps))] * world


def test_reported_failure_ends_the_wait_at_once() -> None:
    store = dist.HashStore()
    a = StepLiveness(store, 0, 2, timeout_s=30.0)
    b = StepLiveness(store, 1, 2, timeout_s=30.0)
    with pytest.raises(ValueError, match="bad input"):
        with b.guard():
            raise ValueError("bad input")
    start = time.monotonic()
    with pytest.raises(RankFailure) as info:
        a.enter(0)
    assert time.monotonic() - start < 5.0
    assert info.value.ranks == [1] and info.value.step == 0
    assert "ValueError: bad input" in info.value.reason
    assert a.failed_ranks() == {1: "ValueError: bad input"}


def test_missing_rank_is_named_after_the_timeout() -> None:
    store = dist.HashStore()
    live = StepLiveness(store, 0, 3, timeout_s=0.3)
    StepLiveness(store, 2, 3).store.set("b200tx/liveness/at/2", "4")  # rank 2 is ahead
    start = time.monotonic()
    with pytest.raises(RankFailure, match="no heartbeat") as info:
        live.enter(4)
    assert 0.3 <= time.monotonic() - start < 5.0
    assert info.value.ranks == [1]


def test_stale_heartbeat_counts_as_missing() -> None:
    store = dist.HashStore()
    a = StepLiveness(store, 0, 2, timeout_s=0.2)
    b = StepLiveness(store, 1, 2, timeout_s=0.2)
    threads = [threading.Thread(target=live.enter, args=(0,)) for live in (a, b)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=10)
    with pytest.raises(RankFailure) as info:
        a.enter(1)  # rank 1 stays at step 0
    assert info.value.ranks == [1] and info.value.step == 1


def test_argument_checks() -> None:
    store = dist.HashStore()
    with pytest.raises(ValueError):
        StepLiveness(store, 2, 2)
    with pytest.raises(ValueError):
        StepLiveness(store, 0, 2, timeout_s=0)


# ---------------------------------------------------------------- gloo ranks


def _worker(rank: int, world: int, port: int, out_dir: str, scenario: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(
        "gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20)
    )
    store = dist.distributed_c10d._get_default_store()
    live = StepLiveness(store, rank, world, timeout_s=1.0)
    result = {"rank": rank}
    leaver = 0 if scenario == "host_exit" else 1
    try:
        for step in range(2):
            live.enter()
            value = torch.ones(4)
            dist.all_reduce(value)
            assert float(value[0]) == world
        if rank == leaver:
            if scenario == "raise":
                try:
                    with live.guard():
                        raise ValueError("bad batch on rank 1")
                except ValueError:
                    result["raised"] = True
                    np.save(os.path.join(out_dir, "rank1.npy"), result)
                    os._exit(0)
            # "exit", "host_exit" and "collective": leave between steps without a word
            os._exit(0)
        start = time.monotonic()
        try:
            if scenario == "collective":
                value = torch.ones(4)
                dist.all_reduce(value)  # the peer is gone: must end with an error
            else:
                live.enter()
            result["error"] = None
        except RankFailure as exc:
            result.update(error="RankFailure", ranks=exc.ranks, reason=exc.reason)
        except Exception as exc:  # noqa: BLE001 - the collective's own error
            result.update(error=type(exc).__name__)
        result["elapsed"] = time.monotonic() - start
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), result)
    finally:
        if rank != leaver:
            abort_process_group()


def _run(scenario: str) -> dict:
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(
            _worker, args=(2, _free_port(), tmp, scenario), nprocs=2, start_method="spawn"
        )
        survivor = 1 if scenario == "host_exit" else 0
        got = np.load(os.path.join(tmp, f"rank{survivor}.npy"), allow_pickle=True).item()
        if scenario == "raise":
            assert np.load(os.path.join(tmp, "rank1.npy"), allow_pickle=True).item()["raised"]
    return got


def test_rank_that_raises_is_reported_before_the_next_step() -> None:
    got = _run("raise")
    assert got["error"] == "RankFailure" and got["ranks"] == [1]
    assert "ValueError: bad batch on rank 1" in got["reason"]
    assert got["elapsed"] < 1.0  # the report, not the timeout, ended the wait


def test_rank_that_exits_silently_is_detected_by_the_heartbeat_timeout() -> None:
    got = _run("exit")
    assert got["error"] == "RankFailure" and got["ranks"] == [1]
    assert "no heartbeat" in got["reason"]
    assert 1.0 <= got["elapsed"] < 10.0


def test_collective_with_a_departed_peer_ends_with_an_error() -> None:
    got = _run("collective")
    assert got["error"] is not None
    assert got["elapsed"] < 25.0  # bounded by the 20 s process-group timeout


def test_store_host_that_exits_is_detected_without_a_hang() -> None:
    # Rank 0 hosts the process group's store; its departure must end the
    # survivor's wait with RankFailure rather than block on the store.
    got = _run("host_exit")
    assert got["error"] == "RankFailure" and got["ranks"] == [0]
    assert got["elapsed"] < 25.0
