"""Failure detection for the data-parallel training exchange.

The reference trains on one GPU and its only failure handling is the stop
flag of the search (src/main.rs:2106-2114); a data-parallel step adds ranks
that can fail.  `StepGuard` keeps a rank from entering a collective that a
dead peer would never join, and keeps a collective that is already in flight
from waiting forever:

* before each step's exchange every rank posts a heartbeat key for that step
  in a TCP key-value store and waits (bounded) for all peers' keys; a peer
  that left between steps is reported as `RankFailure` naming the missing
  ranks, and no collective is launched;
* the exchange itself is issued asynchronously and polled
  (`Work.is_completed`) against a host deadline; on expiry, or when the
  completed work reports an error, the process group is aborted (NCCL
  communicators included) and `RankFailure` is raised.

Everything here runs on the host: no device wait is involved, so a failure
is reported as an exception on every surviving rank instead of a hang.
"""
from __future__ import annotations

import time
from typing import Sequence


class RankFailure(RuntimeError):
    """A peer rank left, or a collective did not complete in time."""

    def __init__(self, msg: str, missing: Sequence[int] = ()):
        super().__init__(msg)
        self.missing = list(missing)


class StepGuard:
    """Heartbeats and bounded collectives for one rank of a data-parallel job.

    `store` is a torch.distributed Store shared by the ranks (for instance a
    TCPStore on MASTER_ADDR); `timeout_s` bounds both the heartbeat wait and
    each collective."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "cnnue/step",
                 group=None):
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = float(timeout_s)
        self.prefix = prefix
        self.group = group

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def arrive(self, step: int) -> None:
        """Posts this rank's heartbeat for `step`."""
        self.store.set(self._key(step, self.rank), b"1")

    def wait_peers(self, step: int) -> None:
        """Waits until every rank posted its heartbeat for `step`; raises
        RankFailure with the missing ranks after `timeout_s`."""
        # polled with the store's non-blocking check: a timed-out blocking
        # wait can leave the client's connection out of step with the server
        deadline = time.monotonic() + self.timeout_s
        missing = [r for r in range(self.world) if r != self.rank]
        while True:
            missing = [r for r in missing if not self.store.check([self._key(step, r)])]
            if not missing:
                return
            if time.monotonic() > deadline:
                raise RankFailure(f"rank {self.rank}: ranks {missing} missed step {step}", missing)
            time.sleep(0.002)

    def all_reduce(self, tensor, step: int, op=None) -> None:
        """Heartbeat, peer check, then an asynchronous all_reduce polled
        against the deadline (abort + RankFailure on expiry or error)."""
        import torch.distributed as dist
        self.arrive(step)
        self.wait_peers(step)
        work = dist.all_reduce(tensor, op=op or dist.ReduceOp.SUM, group=self.group, async_op=True)
        self.wait_work(work, f"all_reduce of step {step}")

    def wait_work(self, work, what: str) -> None:
        deadline = time.monotonic() + self.timeout_s
        while not work.is_completed():
            if time.monotonic() > deadline:
                self.abort()
                raise RankFailure(f"rank {self.rank}: {what} did not complete within {self.timeout_s} s")
            time.sleep(0.0005)
        try:
            work.wait()  # completed: returns at once, or raises the backend's error
        except Exception as e:  # noqa: BLE001 - the backend reports the failure by raising
            self.abort()
            raise RankFailure(f"rank {self.rank}: {what} failed: {e}") from e

    def abort(self) -> None:
        """Aborts the process group (its NCCL communicators included) so that
        nothing waits on it any more; the group must not be used after."""
        import torch.distributed.distributed_c10d as c10d
        try:
            c10d._abort_process_group(self.group or c10d.GroupMember.WORLD)
        except Exception:  # noqa: BLE001 - gloo groups and old versions have no abort: nothing to release
            pass
