"""Data-parallel AZ training on two GPUs (skipped with fewer): two NCCL ranks
each stepping on half of every batch, the mean gradient exchanged, end up
with the same parameters on both ranks, and those of one trainer stepping on
the whole batches up to float32 summation order (as Adam amplifies it)."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _setup():
    from chineseai_b200 import az, az_train
    from tests._azutil import full_policy, trained_like
    w = az.AzWeights.random(64, 20260825)
    trained_like(w, 91)
    full_policy(w, 92)
    s = az_train.random_samples(256, 93)
    return w, s


def _rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist
    from chineseai_b200 import az_train
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    w, s = _setup()
    tr = az_train.AzTrainer(w, lr=2e-3, device=rank, graph=True, group=dist.group.WORLD)
    for k in range(4):
        rows = np.arange(k % 2 * 128, (k % 2 + 1) * 128)
        mine = rows[rank * 64:(rank + 1) * 64]
        tr.step(az_train.pack_batch(s, mine, caps=(40, 96, 96), fixed=True, compact=True))
    out[rank] = [t.copy() for t in tr.tensors()]
    torch.cuda.synchronize()
    del tr
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_data_parallel_equals_full_batch():
    from chineseai_b200 import az_train
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
        assert p.exitcode == 0
    w, s = _setup()
    ref = az_train.AzTrainer(w, lr=2e-3, device=0)
    for k in range(4):
        rows = np.arange(k % 2 * 128, (k % 2 + 1) * 128)
        ref.step(az_train.pack_batch(s, rows, caps=(40, 96, 96), fixed=True, compact=True))
    for a, b in zip(out[0], out[1]):
        np.testing.assert_array_equal(a, b)
    # Adam divides by sqrt(v): a gradient that cancels to ~0 over the whole
    # batch but not in the two half sums becomes a step of up to lr.  Every
    # element stays within 4 steps x lr; nearly all agree to 1e-4.
    lr = 2e-3
    for a, r in zip(out[0], ref.tensors()):
        d = np.abs(a.astype(np.float64) - r)
        assert d.max() <= 4 * lr * 1.01
        loose = d > 1e-6 + 1e-4 * np.abs(r)
        assert loose.mean() <= 1e-4, loose.sum()


def _rank_bad(rank, world, port, out):
    import datetime

    import torch.distributed as dist
    from chineseai_b200 import az_train
    from chineseai_b200._lib import CnnueError
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    w, s = _setup()
    tr = az_train.AzTrainer(w, lr=2e-3, device=rank, graph=False, group=dist.group.WORLD)
    before = [t.copy() for t in tr.tensors()]
    b = az_train.pack_batch(s, np.arange(rank * 64, (rank + 1) * 64), caps=(40, 96, 96), fixed=True, compact=True)
    if rank == 1:
        b.policy_items[0, 0] = (3000 | 1 << 47)  # a move index past the 2086-move space
    raised = False
    try:
        tr.step(b)
    except CnnueError:
        raised = True
    unchanged = all(np.array_equal(a, c) for a, c in zip(before, tr.tensors()))
    # the group is still usable: a clean step on both ranks goes through
    tr.step(az_train.pack_batch(s, np.arange(128 + rank * 64, 128 + (rank + 1) * 64), caps=(40, 96, 96),
                                fixed=True, compact=True))
    out[rank] = (raised, unchanged)
    torch.cuda.synchronize()
    del tr
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_bad_batch_on_one_rank_stops_every_rank():
    """Rank 1's batch holds a bad move index: both ranks raise after the
    step, neither applies AdamW (parameters unchanged), and the next clean
    step runs on both."""
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_bad, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
        assert p.exitcode == 0
    assert out[0] == (True, True) and out[1] == (True, True)
