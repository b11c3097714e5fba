"""CPU tests of the utterance-parallel sharding (the multi-GPU path).

World-size-2 gloo process groups stand in for GPUs: every rank computes the
plan locally, the ranks check over gloo that together they cover every
utterance exactly once, and a rank that dies is detected on the host (it
never posts its heartbeat to the store) and its work re-queued -- no GPU is
faulted or hung.
"""
from __future__ import annotations

import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from ovnative_b200 import shard as S


def test_lpt_plan_is_balanced_and_complete():
    lengths = S.synthetic_utterances()
    for world in (1, 2, 4, 8):
        plan = S.lpt_assign(lengths, world)
        ids = sorted(i for p in plan for i in p)
        assert ids == list(range(len(lengths)))
        loads = S.plan_loads(lengths, plan)
        assert max(loads) / (sum(loads) / world) < 1.10  # within 10% of perfect


def test_requeue_moves_only_unfinished_work():
    lengths = S.synthetic_utterances(n=20, seed=3)
    plan = S.lpt_assign(lengths, 4)
    done = set(plan[2][:2])
    new = S.requeue(lengths, plan, dead={2}, done=done)
    assert new[2] == []
    moved = set(plan[2]) - done
    got = [i for r in (0, 1, 3) for i in new[r]]
    assert moved <= set(got)
    assert sorted(got + sorted(done)) == list(range(20))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lengths, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0,
                          timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        plan = S.lpt_assign(lengths, world)
        mine = plan[rank]
        got = [None] * world
        dist.all_gather_object(got, mine)
        flat = sorted(i for p in got for i in p)
        ok = flat == list(range(len(lengths))) and got == plan
        if rank == fail_rank:
            # Leave between steps: post nothing, exit without the heartbeat.
            q.put((rank, ok, None))
            return
        store.set(f"done/{rank}", ",".join(map(str, mine)))
        done = set(mine)
        dead = set()
        if rank == 0 and fail_rank is not None:
            deadline = time.time() + 5
            while time.time() < deadline and not store.check([f"done/{fail_rank}"]):
                time.sleep(0.05)
            if not store.check([f"done/{fail_rank}"]):
                dead.add(fail_rank)
            new = S.requeue(lengths, plan, dead, done=set())
            done |= set(new[0])
        q.put((rank, ok, sorted(done) if rank == 0 else None))
    finally:
        if fail_rank is None:
            dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [None, 1])
def test_gloo_world2_shard_and_failure(fail_rank):
    lengths = [int(x) for x in S.synthetic_utterances(n=16, seed=5)]
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, lengths, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, ok, done = q.get(timeout=60)
        results[r] = (ok, done)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert all(ok for ok, _ in results.values())
    if fail_rank is not None:
        # rank 0 detected the silent rank and finished its utterances too
        assert results[0][1] == list(range(len(lengths)))
