"""Data-parallel replicas: one engine per GPU, requests routed by the host.

ASR requests are independent, so scaling across GPUs needs no collective on the data
path: each rank runs its own ``AsrEngine`` (own weights, KV pool and graphs) over the
requests routed to it. ``torch.distributed`` is used only to start together and to
combine timings (max over ranks) and totals (sum over ranks). NCCL on GPUs; gloo when
the group runs on CPU (the multi-process tests).
"""

from __future__ import annotations

import heapq
import os
from datetime import timedelta


def rank_env() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the torchrun environment (1 process: 0, 1, 0)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def route_by_duration(durations, world: int) -> list[list[int]]:
    """Split request indices over ``world`` replicas so their audio seconds balance:
    longest first, each to the replica with the least audio so far (ties: lowest rank).
    Every index appears exactly once; each replica's list is in input order."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0.0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(durations)), key=lambda j: (-float(durations[j]), j)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + float(durations[i]), r))
    return [sorted(x) for x in out]


class ReplicaGroup:
    """Process group of the replicas (no-op for a single process).

    ``backend`` "nccl" pins each rank to GPU ``local_rank``; "gloo" keeps tensors on the
    CPU. The group's timeout bounds how long a rank waits for one that never arrives.
    """

    def __init__(self, backend: str = "nccl", timeout_s: float = 600.0):
        import torch

        self.torch = torch
        self.rank, self.world, self.local = rank_env()
        self.backend = backend
        self.pg = None
        if self.world > 1:
            import torch.distributed as dist

            kwargs = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                kwargs["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kwargs)
            self.pg = dist

    def _tensor(self, value: float):
        dev = "cuda" if self.backend == "nccl" else "cpu"
        return self.torch.tensor([float(value)], dtype=self.torch.float64, device=dev)

    def barrier(self) -> None:
        if self.pg is not None:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return float(value)
        t = self._tensor(value)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self.pg is None:
            return float(value)
        t = self._tensor(value)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def gather(self, values: list[int]) -> list[list[int]]:
        """All ranks' integer lists (for routing checks)."""
        if self.pg is None:
            return [list(values)]
        out: list = [None] * self.world
        self.pg.all_gather_object(out, list(values))
        return out

    def close(self) -> None:
        if self.pg is not None:
            self.pg.destroy_process_group()
            self.pg = None


def throughput(group: ReplicaGroup, seconds_of_audio: float, elapsed_ms: float) -> tuple[float, float]:
    """Whole-job audio-s/s: every rank's audio over the slowest rank's time."""
    ms_max = group.max(elapsed_ms)
    return group.sum(seconds_of_audio) / (ms_max / 1000.0), ms_max
