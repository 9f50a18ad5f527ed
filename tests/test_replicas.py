"""Data-parallel replicas on CPU: world_size-2 gloo groups (no GPU).

The multi-GPU path has no collective on its data path; what runs across ranks is the
start barrier, the max-over-ranks timing and the sum of work, plus the host router that
splits a shared request list. These run here as two gloo processes.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from voiceagent_b200.replicas import (ReplicaGroup, pin_host_cores, route_by_duration,
                                      throughput, transcribe_share)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank: int, world: int, port: int) -> None:
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))


def _worker(rank: int, world: int, port: int, durations, results) -> None:
    _env(rank, world, port)
    g = ReplicaGroup("gloo", timeout_s=30)
    try:
        assert (g.rank, g.world) == (rank, world)
        # every rank routes the same list; its own share is its slice
        shares = route_by_duration(durations, world)
        mine = shares[rank]
        gathered = g.gather(mine)
        audio = float(np.sum(np.asarray(durations)[mine]))
        elapsed_ms = 100.0 * (rank + 1)  # rank 1 is the slow one
        g.barrier()
        value, ms_max = throughput(g, audio, elapsed_ms)
        results.put((rank, gathered, value, ms_max, g.max(rank), g.sum(1.0)))
    finally:
        g.close()


def test_two_gloo_replicas_combine_timings_and_route_consistently():
    durations = list(np.random.default_rng(0).lognormal(np.log(7.0), 0.6, size=37))
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, durations, results)) for r in range(2)]
    for p in procs:
        p.start()
    out = [results.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    total = sum(durations)
    for rank, gathered, value, ms_max, rmax, rsum in out:
        assert ms_max == 200.0 and rmax == 1.0 and rsum == 2.0
        assert value == pytest.approx(total / 0.2)  # all audio over the slowest rank's time
        flat = sorted(i for share in gathered for i in share)
        assert flat == list(range(len(durations)))  # a partition, identical on both ranks
    assert out[0][1] == out[1][1]


def _leaver(rank: int, world: int, port: int, results) -> None:
    _env(rank, world, port)
    g = ReplicaGroup("gloo", timeout_s=5)
    if rank == 1:
        g.close()  # leaves between steps, never reaches the barrier
        return
    try:
        g.barrier()
        results.put("joined")
    except Exception as e:  # noqa: BLE001 - the failure is what this test checks
        results.put(type(e).__name__)


def test_rank_that_leaves_ends_the_others_barrier_with_an_error():
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    outcome = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert outcome != "joined"


def test_router_balances_audio_seconds():
    d = list(np.random.default_rng(1).lognormal(np.log(7.0), 0.6, size=512))
    for world in (1, 2, 4, 8):
        shares = route_by_duration(d, world)
        loads = [sum(d[i] for i in s) for s in shares]
        assert sorted(i for s in shares for i in s) == list(range(512))
        assert max(loads) - min(loads) <= max(d)  # greedy LPT bound


def test_reference_arm_is_rank_zero_only(monkeypatch, capsys):
    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    args = type("Args", (), {"clips": 4, "warmup": 0, "steps": 1, "preset": "tiny",
                             "decode_tokens": 2, "gpus": 2})()
    bench.run_reference_arm(args)  # rank 1 of 2: exits without work or output
    assert capsys.readouterr().out == ""


def _shared_job_worker(rank: int, world: int, port: int, results) -> None:
    from voiceagent_b200.workload import SAMPLE_RATE, Job

    _env(rank, world, port)
    g = ReplicaGroup("gloo", timeout_s=30)
    try:
        cores = pin_host_cores(rank, world)
        job = Job("config4")  # 4096 clips + a 20-minute file in 30 s chunks
        # stand-in transcriber: one output per request, here the sample count it got
        done = transcribe_share(g, job, lambda waves: [len(w) for w in waves], batch=512)
        ok = all(n == int(round(job.durations[i] * SAMPLE_RATE)) for i, n in done.items())
        audio = float(sum(job.durations[i] for i in done))
        results.put((rank, sorted(done), ok, g.gather(cores), g.sum(audio),
                     float(job.durations.sum())))
    finally:
        g.close()


def test_two_gloo_replicas_transcribe_a_routed_job_exactly_once():
    """One shared job (config 4's 4136 requests) split by the host router over two gloo
    ranks, each pinned to its own host cores: every request is transcribed exactly once,
    each rank synthesises the right waveform for each of its requests, and the summed
    audio is the job's."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_shared_job_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(results.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shares = [set(o[1]) for o in out]
    assert not shares[0] & shares[1]
    assert sorted(shares[0] | shares[1]) == list(range(4136))
    assert all(o[2] for o in out)
    assert out[0][4] == pytest.approx(out[0][5])  # all audio accounted for, once
    cores = out[0][3]
    if len(os.sched_getaffinity(0)) >= 2:
        assert cores[0] and cores[1] and not set(cores[0]) & set(cores[1])
