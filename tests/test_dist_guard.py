"""Failure detection of the data-parallel exchange on CPU (gloo ranks): a
rank that leaves between steps is reported on every surviving rank as
RankFailure naming it, before any collective is launched, instead of a hang;
the steps before the failure reduce normally."""
import os
import time

import torch
import torch.multiprocessing as mp

from chineseai_b200.dist_guard import RankFailure, StepGuard


def _rank(rank, world, port, leave_at, out):
    import datetime

    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    guard = StepGuard(store, rank, world, timeout_s=2.0)
    sums = []
    result = "ok"
    t0 = time.monotonic()
    try:
        for step in range(4):
            if rank == world - 1 and step == leave_at:
                result = "left"
                break
            x = torch.full((4,), float(rank + 1))
            guard.all_reduce(x, step)
            sums.append(float(x[0]))
    except RankFailure as e:
        result = ("failure", e.missing)
    out[rank] = (result, sums, time.monotonic() - t0)
    if result == "left":
        os._exit(0)  # leave without a word to the group
    os._exit(0)


def test_rank_leaving_between_steps_is_reported_not_hung():
    world, leave_at = 3, 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 31000 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, world, port, leave_at, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for r in range(world - 1):
        result, sums, took = out[r]
        assert result == ("failure", [world - 1]), result
        assert sums == [6.0, 6.0]  # steps 0 and 1 reduced over all three ranks
        assert took < 30
    assert out[world - 1][0] == "left"
