"""Host-side failure detection for the expert-parallel decode loop (one process per GPU).

The reference reports failures as status phases of its server and loader threads
(src/duplex/server.py:76-82, src/duplex/fast_engine.py:64-73); it has no multi-GPU
path.  The expert-parallel layer (duplex.streaming.ep_moe) adds collectives, and with
them the failure a single process never sees: a rank that leaves.  Two guards, both on
the host, neither needing a GPU fault to test:

* `Heartbeat` -- step-gated liveness through the process group's store.  Before a rank
  launches step s it calls `ready(s)`: it posts its own key for s and waits, under a
  host timeout, until every rank has posted s.  A rank that exited, crashed or stopped
  stepping makes the others raise `PeerLost` there, BEFORE they launch any kernel or
  collective of step s, so no collective ever waits on a peer that is gone.
* `guard_step` -- waits for the step's completion event on the host under a timeout.
  On expiry it aborts the group's communicators (ncclCommAbort through torch, which
  also stops collectives in flight) and raises `StepTimeout`.  torch's NCCL watchdog
  additionally polls the communicators' asynchronous errors and aborts a collective that
  outlives the group's timeout (duplex.benchutil.init_nccl).
"""

from __future__ import annotations

import time
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.distributed.distributed_c10d as c10d


class PeerLost(RuntimeError):
    """A rank did not reach the step within the heartbeat timeout."""


class StepTimeout(RuntimeError):
    """A step's work did not complete within the host timeout; the group was aborted."""


class Heartbeat:
    """Step-gated liveness of the ranks of `group` through its store.

    timeout_s bounds every wait; keys older than two steps are deleted as ranks move on,
    so the store holds O(world) keys whatever the number of steps.
    """

    def __init__(self, timeout_s: float = 5.0, group=None, prefix: str = "duplex-hb"):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = float(timeout_s)
        base = c10d._get_process_group_store(group) if group is not None else c10d._get_default_store()
        self.store = dist.PrefixStore(prefix, base)

    def _key(self, rank: int, step: int) -> str:
        return f"{rank}/{step}"

    def ready(self, step: int) -> None:
        """Post this rank's step and wait until every rank has posted it (PeerLost if not)."""
        self.store.set(self._key(self.rank, step), "1")
        others = [self._key(r, step) for r in range(self.world) if r != self.rank]
        if others:
            try:
                self.store.wait(others, timedelta(seconds=self.timeout_s))
            except Exception as e:  # the store raises on timeout, or when its host is gone
                missing = []
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    try:
                        if not self.store.check([self._key(r, step)]):
                            missing.append(r)
                    except Exception:
                        missing.append(r)
                raise PeerLost(f"rank {self.rank}: ranks {missing} did not reach step {step} "
                               f"within {self.timeout_s:.1f} s") from e
        if step >= 2:
            try:
                self.store.delete_key(self._key(self.rank, step - 2))
            except Exception:  # a store without deletion keeps the key: harmless
                pass


def abort_group(group=None) -> None:
    """Abort the communicators of `group` (ncclCommAbort for NCCL); the group is unusable
    afterwards."""
    c10d._abort_process_group(group if group is not None else c10d.GroupMember.WORLD)


def guard_step(timeout_s: float, stream=None, group=None, poll_s: float = 1e-4) -> float:
    """Wait on the host for the work queued so far on `stream` (default: the current
    stream), at most timeout_s seconds.  Returns the seconds waited; on expiry aborts
    `group` and raises StepTimeout."""
    ev = torch.cuda.Event()
    ev.record(stream)
    t0 = time.monotonic()
    while not ev.query():
        if time.monotonic() - t0 > timeout_s:
            abort_group(group)
            raise StepTimeout(f"step did not complete within {timeout_s:.2f} s; "
                              "communicators aborted")
        time.sleep(poll_s)
    return time.monotonic() - t0
