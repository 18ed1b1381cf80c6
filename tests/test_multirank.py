"""Replica host logic on CPU with gloo, world size 2 (no GPU): sharding covers
every stream once, the timing reduction takes the slowest rank, and a rank that
leaves makes the other's next collective fail within the group timeout."""

from __future__ import annotations

import importlib
import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import PACKAGE, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_covers_every_unit_once(lffw):
    replicas = importlib.import_module(PACKAGE + ".replicas")
    for units in (0, 1, 7, 64, 128, 129):
        for world in (1, 2, 3, 4, 8):
            got = [u for r in range(world) for u in replicas.shard(units, r, world)]
            assert got == list(range(units))
            sizes = [len(replicas.shard(units, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)
    assert replicas.whole_job_rate(10.0, 4, 2.0) == 20.0


def _worker(rank, world, port, queue, leave_early):
    import sys

    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    replicas = importlib.import_module(PACKAGE + ".replicas")
    dist = replicas.init("gloo", timeout_s=10.0)
    try:
        mine = list(replicas.shard(128, rank, world))
        worst = replicas.max_over_ranks([1.0 + rank, 5.0 - rank], dist)
        dist.barrier()
        if leave_early and rank == 1:
            queue.put((rank, mine, worst, "left"))
            return  # leaves between steps, with nothing in flight
        status = "ok"
        if leave_early:
            try:
                replicas.max_over_ranks([0.0], dist)
                status = "no error"
            except Exception:  # the peer is gone: the collective fails instead of hanging
                status = "peer gone"
        queue.put((rank, mine, worst, status))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, leave_early):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue, leave_early)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_two_ranks_shard_and_reduce():
    results = _run(2, leave_early=False)
    assert [r[0] for r in results] == [0, 1]
    assert results[0][1] + results[1][1] == list(range(128))
    assert all(r[2] == [2.0, 5.0] for r in results)  # element-wise max over ranks
    assert all(r[3] == "ok" for r in results)


def test_rank_leaving_fails_the_next_collective():
    results = _run(2, leave_early=True)
    assert results[1][3] == "left"
    assert results[0][3] == "peer gone"
