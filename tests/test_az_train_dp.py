"""Data-parallel AZ training without a GPU: the exchange (mean all-reduce of
the flat gradient) on two gloo ranks, and the identity it relies on - the
mean of the two half-batch gradients of the reference loss (float64
restatement of compute_batch_loss) is the whole batch's gradient."""
import os

import numpy as np
import torch
import torch.multiprocessing as mp

from chineseai_b200 import az, az_train
from oracle import az_train_ref
from tests._azutil import full_policy, trained_like


def _rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.arange(10, dtype=torch.float32) * (rank + 1)
    w = az_train.mean_allreduce_(g)
    out[rank] = (w, g.tolist())
    dist.destroy_process_group()


def test_mean_allreduce_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    want = (np.arange(10) * 1.5).tolist()
    assert out[0] == (2, want) and out[1] == (2, want)


def test_half_batch_gradients_average_to_full_batch():
    w = az.AzWeights.random(32, 20260823)
    trained_like(w, 81)
    full_policy(w, 82)
    s = az_train.random_samples(64, 83)
    full = az_train.pack_batch(s, caps=(40, 96, 96), fixed=True)
    halves = [az_train.pack_batch(s, np.arange(k * 32, (k + 1) * 32), caps=(40, 96, 96), fixed=True)
              for k in range(2)]
    _, gf = az_train_ref.gradients(w.tensors(), full)
    _, g0 = az_train_ref.gradients(w.tensors(), halves[0])
    _, g1 = az_train_ref.gradients(w.tensors(), halves[1])
    for a, b, c in zip(gf, g0, g1):
        np.testing.assert_allclose((b + c) / 2, a, rtol=1e-9, atol=1e-12)


def _rank_status(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    tail_at, n_grad = 16, 10
    buf = torch.zeros(tail_at + 64)
    buf[:n_grad] = torch.arange(10, dtype=torch.float32) * (rank + 1)
    metrics = torch.arange(30, dtype=torch.float32) + 100 * rank
    word = 1 if rank == 1 else 0  # rank 1's batch had a bad index
    m, w = az_train.exchange_with_status_(buf, n_grad, tail_at, metrics, word)
    out[rank] = (buf[:n_grad].tolist(), m.tolist(), w)
    dist.destroy_process_group()


def test_exchange_reduces_status_and_metrics_across_ranks():
    """A bad batch on one rank: both ranks read the same status word (so
    both skip AdamW and raise together), the metrics are the sums over the
    ranks, the gradient their mean."""
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29500 + (os.getpid() + 7) % 1000
    procs = [ctx.Process(target=_rank_status, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(2):
        g, m, w = out[r]
        assert w == 1
        np.testing.assert_allclose(g, np.arange(10) * 1.5)
        np.testing.assert_allclose(m, 2 * np.arange(30) + 100)
