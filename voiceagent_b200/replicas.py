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


def share_of(durations, group: "ReplicaGroup") -> list[int]:
    """This rank's request indices of a job routed by :func:`route_by_duration` (every
    rank computes the same routing from the same durations, so no message is needed)."""
    return route_by_duration(durations, group.world)[group.rank]


def transcribe_share(group: "ReplicaGroup", job, transcribe, batch: int) -> dict[int, object]:
    """Run this rank's share of ``job`` (``job.durations``, ``job.waveforms(indices)``)
    through ``transcribe(waveforms) -> outputs`` in slices of ``batch`` requests, waveforms
    synthesised per slice. Returns {request index: output} for the indices routed here."""
    mine = share_of(job.durations, group)
    out: dict[int, object] = {}
    for i in range(0, len(mine), batch):
        idx = mine[i:i + batch]
        for j, o in zip(idx, transcribe(job.waveforms(idx))):
            out[j] = o
    return out


def pin_host_cores(local_rank: int, local_world: int) -> list[int]:
    """Restrict this process to its own slice of the host cores and size torch's
    intra-op pool to it.

    Each replica's scheduler, packer calls, graph launches and frontend copies are host
    work; with one process per GPU on the same node, unpinned processes contend for the
    same cores. The cores this process may use are split into ``local_world`` equal,
    disjoint slices (in id order) and rank ``local_rank`` keeps slice ``local_rank``;
    when there are fewer cores than ranks the slices overlap instead (every rank keeps
    at least one core). Returns the cores kept."""
    import torch

    if not hasattr(os, "sched_getaffinity"):
        return []
    cores = sorted(os.sched_getaffinity(0))
    if local_world <= 1 or not cores:
        return cores
    per = len(cores) // local_world
    mine = (cores[local_rank * per:(local_rank + 1) * per] if per >= 1
            else [cores[local_rank % len(cores)]])
    os.sched_setaffinity(0, mine)
    torch.set_num_threads(len(mine))
    return mine


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
