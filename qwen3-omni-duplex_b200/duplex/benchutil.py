"""Helpers of the benchmark harness: rank plumbing, max-over-ranks timing, clock sampling."""

from __future__ import annotations

import os
import statistics
import subprocess
import threading
from datetime import timedelta

import torch
import torch.distributed as dist


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(backend: str, timeout_s: int = 120):
    ws, rank, _ = dist_env()
    if ws > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))
    return ws, rank


def init_nccl(device, timeout_s: int = 180):
    """NCCL process group of the torchrun ranks (a group of one when not launched by
    torchrun), with a `timeout_s` collective timeout: torch's watchdog polls the
    communicators' asynchronous errors (ncclCommGetAsyncError) and aborts a communicator
    whose collective outlives the timeout, so a rank that dies makes the others' next
    collective fail instead of hanging.  duplex.health adds the host-side guards: a
    heartbeat that finds a departed rank before the next launch, and a step guard that
    aborts the group.  The communicators are blocking: with `config.blocking = 0` this
    torch build's all-to-all raised "NCCL Error 7: operation in progress" on 2 and 4 B200s.
    """
    import socket
    if "WORLD_SIZE" not in os.environ:
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
        s.close()
        os.environ.update(WORLD_SIZE="1", RANK="0", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=timeout_s))
    # set the communicator up with one collective now, before any stream capture begins
    t = torch.ones(1, device=device)
    dist.all_reduce(t)
    torch.cuda.synchronize(device)
    return dist.get_world_size(), dist.get_rank()


def barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def soak_replays(seconds: float, one_replay_s: float, device=None) -> int:
    """How many replays of a step fill about `seconds`, given one replay's time on this
    rank.  The count is the same on every rank (from the max over ranks of the replay
    time), which a step that exchanges with the other ranks requires: a rank that
    replayed once more than its peers would wait on exchanges that never come."""
    t = max_over_ranks(one_replay_s, device)
    return max(1, int(seconds / max(t, 1e-6))) if seconds > 0 else 0


QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """nvidia-smi sampling (every `ms`) of SM clock and throttle reasons while a
    workload runs; `summary()` gives median SM MHz, max MHz and active reasons."""

    def __init__(self, indices=None, ms: int = 100):
        self.indices, self.ms = indices, ms
        self.rows, self.proc, self.thread = [], None, None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               "-lms", str(self.ms)]
        if self.indices:
            cmd += ["-i", ",".join(str(i) for i in self.indices)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        return self

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in self.rows if r[3].replace(".", "").isdigit()]
        active = sorted({name for r in self.rows for name, v in zip(REASONS, r[5:9])
                         if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None,
                "reasons": active, "samples": len(self.rows)}


def visible_gpu_indices(n: int):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if all(i.isdigit() for i in ids):
            return [int(i) for i in ids[:n]]
    return list(range(n))
