"""Host-side failure detection between the steps of a multi-process run.

The reference is single-GPU; its failure handling is host-side (a spawned
process per measurement whose errors are marshalled back,
benchmarking/device_isolation.py:151-203, and infeasible-vs-infrastructure
classification, autotune/evaluation.py:142).  The multi-GPU runtimes here
add the one failure the reference cannot have: a rank of a process group
that raises, exits or stops answering.

`StepLiveness` detects it on the host, before the next launch, through the
process group's key-value store:

* ``enter(step)`` announces that this rank reached the start of ``step`` and
  waits until every rank has announced it.  A rank that reported a failure
  ends the wait at once; a rank that never arrives ends it after
  ``timeout_s``; a store that stops answering (the rank hosting it died) ends
  it with the ranks not yet seen.  Either way ``RankFailure`` names the ranks and no kernel or
  collective of ``step`` is launched by the survivors, so none of them waits
  on the GPU for a peer that is gone (the peer-reduction LayerNorm polls its
  peers' flags; a collective would wait for the process-group timeout).
* ``guard()`` wraps this rank's host work of a step: an exception inside it is
  reported to the store (``report``) before it propagates, so the peers learn
  of it at their next ``enter`` instead of after a timeout.

A rank therefore leaves only between steps, with nothing of its own in
flight on the GPU.  The process group's own timeout stays the last bound for
a failure inside a step (a collective whose peer died mid-step ends with an
error after that timeout).
"""

from __future__ import annotations

import contextlib
import time
from collections.abc import Iterator


class RankFailure(RuntimeError):
    """One or more ranks failed or stopped answering before ``step``."""

    def __init__(self, ranks: list[int], step: int, reason: str) -> None:
        self.ranks = ranks
        self.step = step
        self.reason = reason
        super().__init__(f"rank(s) {ranks} failed before step {step}: {reason}")


class StepLiveness:
    """Step-boundary liveness of ``world`` ranks over a c10d store.

    ``store`` is any ``torch.distributed.Store`` (the default group's store:
    ``torch.distributed.distributed_c10d._get_default_store()``, or a
    ``TCPStore``); ``prefix`` separates independent users of one store.
    Keys: ``<prefix>/at/<rank>`` holds the last step the rank entered;
    ``<prefix>/failed/<rank>`` the reason of a reported failure, counted in
    ``<prefix>/failures``.
    """

    def __init__(
        self,
        store: object,
        rank: int,
        world: int,
        *,
        timeout_s: float = 5.0,
        poll_s: float = 0.002,
        prefix: str = "b200tx/liveness",
    ) -> None:
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} is not in a world of {world}")
        if timeout_s <= 0 or poll_s <= 0:
            raise ValueError("timeout_s and poll_s must be positive")
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = float(timeout_s)
        self.poll_s = float(poll_s)
        self.prefix = prefix
        self.step = -1

    def _key(self, *parts: object) -> str:
        return "/".join((self.prefix, *map(str, parts)))

    def report(self, reason: str) -> None:
        """Record that this rank failed (seen by the peers' next ``enter``)."""

        self.store.set(self._key("failed", self.rank), reason[:512])
        self.store.add(self._key("failures"), 1)

    def failed_ranks(self) -> dict[int, str]:
        """Ranks that reported a failure, with their reasons."""

        if self.store.add(self._key("failures"), 0) == 0:
            return {}
        out: dict[int, str] = {}
        for r in range(self.world):
            key = self._key("failed", r)
            if self.store.check([key]):
                out[r] = self.store.get(key).decode("utf-8", "replace")
        return out

    def _at(self, r: int) -> int:
        key = self._key("at", r)
        if not self.store.check([key]):
            return -1
        return int(self.store.get(key))

    def enter(self, step: int | None = None) -> int:
        """Announce ``step`` (default: the next one) and wait for every rank.

        Returns the step.  Raises ``RankFailure`` as soon as a rank reports a
        failure, or when ranks have not arrived within ``timeout_s``.
        """

        step = self.step + 1 if step is None else int(step)
        self.step = step
        deadline = time.monotonic() + self.timeout_s
        waiting = [r for r in range(self.world) if r != self.rank]
        try:
            self.store.set(self._key("at", self.rank), str(step))
            while True:
                failed = self.failed_ranks()
                if failed:
                    ranks = sorted(failed)
                    raise RankFailure(ranks, step, "; ".join(f"rank {r}: {failed[r]}" for r in ranks))
                waiting = [r for r in waiting if self._at(r) < step]
                if not waiting:
                    return step
                if time.monotonic() > deadline:
                    raise RankFailure(waiting, step, f"no heartbeat within {self.timeout_s:g} s")
                time.sleep(self.poll_s)
        except RankFailure:
            raise
        except Exception as exc:  # noqa: BLE001 - the store itself is gone (its host rank died)
            raise RankFailure(waiting, step, f"store unreachable: {type(exc).__name__}: {exc}") from exc

    @contextlib.contextmanager
    def guard(self) -> Iterator[None]:
        """Report an exception raised by this rank's step before re-raising it."""

        try:
            yield
        except RankFailure:
            raise
        except BaseException as exc:
            with contextlib.suppress(Exception):
                self.report(f"{type(exc).__name__}: {exc}")
            raise


def abort_process_group(group: object | None = None) -> None:
    """Tear down a process group after a ``RankFailure``.

    Uses the c10d abort where this PyTorch has one (it does not wait for the
    failed peer), else ``destroy_process_group``.  Call it only with none of
    this rank's collectives in flight.
    """

    import torch.distributed as dist

    if not dist.is_initialized():
        return
    abort = getattr(dist.distributed_c10d, "_abort_process_group", None)
    if abort is not None:
        try:
            abort(group) if group is not None else abort()
            return
        except Exception:  # noqa: BLE001 - fall back to the plain teardown
            pass
    dist.destroy_process_group(group)


__all__ = ["RankFailure", "StepLiveness", "abort_process_group"]
