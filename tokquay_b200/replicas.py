"""Replica-parallel plumbing: one decode engine and KV pool per GPU.

The reference has no multi-device path (its engine owns one model and one
``BlockAllocator``; tokquay/engine.py:31-63).  Paged attention does not shard
across GPUs without a collective on the data path, so N GPUs run N
independent replicas, each decoding its own sequences out of its own pool.
The only cross-rank traffic is host-side bookkeeping: a barrier around the
timed region and the reduction of per-rank times and token counts.

Whole-job throughput is ``sum(tokens over ranks) / max(time over ranks)``:
the job is done when its slowest replica is.

The helpers work on any process-group backend: tensors live on the current
CUDA device under NCCL and on the host under gloo.
"""

from __future__ import annotations

import datetime
import os

import torch

__all__ = [
    "ReplicaInfo",
    "setup",
    "teardown",
    "barrier",
    "max_over_ranks",
    "sum_over_ranks",
    "all_over_ranks",
    "whole_job_rate",
    "replica_seed",
]


class ReplicaInfo:
    """Rank layout read from the launcher's environment (torchrun sets
    ``WORLD_SIZE``, ``RANK`` and ``LOCAL_RANK``)."""

    def __init__(self, world: int, rank: int, local: int):
        if world < 1 or not (0 <= rank < world) or local < 0:
            raise ValueError(f"bad rank layout: world={world} rank={rank} local={local}")
        self.world, self.rank, self.local = world, rank, local

    @classmethod
    def from_env(cls, env=None) -> "ReplicaInfo":
        env = os.environ if env is None else env
        return cls(int(env.get("WORLD_SIZE", "1")), int(env.get("RANK", "0")), int(env.get("LOCAL_RANK", "0")))

    def __repr__(self):
        return f"ReplicaInfo(world={self.world}, rank={self.rank}, local={self.local})"


def _dist():
    import torch.distributed as dist

    return dist


def setup(backend: str | None = None, timeout_s: float = 600.0, info: ReplicaInfo | None = None) -> ReplicaInfo:
    """Bind this process to its GPU and, for world > 1, join the process group.

    ``backend`` defaults to ``nccl`` when CUDA is available, else ``gloo``.
    The timeout bounds every host collective, so a rank that dies makes the
    others fail instead of waiting for good."""
    info = info or ReplicaInfo.from_env()
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(info.local)
    if info.world > 1:
        dist = _dist()
        backend = backend or ("nccl" if cuda else "gloo")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", info.local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return info


def teardown(info: ReplicaInfo) -> None:
    if info.world > 1:
        dist = _dist()
        if dist.is_initialized():
            dist.destroy_process_group()


def _device():
    dist = _dist()
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def barrier(world: int) -> None:
    if world > 1:
        _dist().barrier()


def _reduce(x: float, world: int, op) -> float:
    if world == 1:
        return float(x)
    dist = _dist()
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, _dist().ReduceOp.MAX if world > 1 else None)


def sum_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, _dist().ReduceOp.SUM if world > 1 else None)


def all_over_ranks(x: float, world: int) -> list[float]:
    """Every rank's ``x``, in rank order (the spread behind a max over ranks)."""
    if world == 1:
        return [float(x)]
    dist = _dist()
    t = torch.zeros(world, dtype=torch.float64, device=_device())
    t[dist.get_rank()] = float(x)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(v) for v in t.tolist()]


def whole_job_rate(units: float, seconds: float, world: int) -> tuple[float, float, float]:
    """(units of all ranks, slowest rank's seconds, units/second of the job)."""
    total = sum_over_ranks(units, world)
    slowest = max_over_ranks(seconds, world)
    return total, slowest, (total / slowest if slowest > 0 else float("nan"))


def replica_seed(base: int, rank: int) -> int:
    """Each replica decodes its own sequences: the workload seed of a rank."""
    return base + rank
