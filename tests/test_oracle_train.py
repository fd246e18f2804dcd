"""CPU tests of the training-step oracle: its hand-written backward against
torch autograd, Adam against a direct restatement, and the data-parallel
gradient exchange (sum all-reduce / world) over two gloo ranks."""
import os

import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import synth, train
from tests import _torchref


@pytest.fixture(scope="module")
def params():
    return train.init_params(3)


def test_oracle_gradient_matches_autograd(params):
    pos = synth.positions(12, 5)
    t = train.targets(12, 6)
    st, loss, g = oracle.t_grad(params, pos, t)
    assert st == 0
    ref_loss, ref_g = _torchref.loss_and_grad(params, pos, t)
    assert abs(loss - ref_loss) <= 1e-6 * max(1.0, abs(ref_loss))
    gs, rs = train.split(g), train.split(ref_g)
    for name, _ in train.LAYOUT:
        scale = np.abs(rs[name]).max()
        assert scale > 0, name
        np.testing.assert_allclose(gs[name], rs[name], rtol=1e-4, atol=1e-5 * scale, err_msg=name)


def test_oracle_adam_matches_published_update():
    rng = np.random.default_rng(0)
    w = rng.normal(size=1000).astype(np.float32)
    m = np.zeros(1000, np.float32)
    v = np.zeros(1000, np.float32)
    w0, m0, v0 = w.copy(), m.copy(), v.copy()
    for step in (1, 2, 3):
        g = rng.normal(size=1000).astype(np.float32)
        oracle.adam(w, m, v, g, 0.5, 1e-3, 0.9, 0.999, 1e-8, step)
        gg = g.astype(np.float64) * 0.5
        m0 = 0.9 * m0 + 0.1 * gg
        v0 = 0.999 * v0 + 0.001 * gg * gg
        w0 = w0 - 1e-3 * (m0 / (1 - 0.9 ** step)) / (np.sqrt(v0 / (1 - 0.999 ** step)) + 1e-8)
    np.testing.assert_allclose(w, w0, rtol=1e-5, atol=1e-6)


def _dp_rank(rank, world, port, params, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pos = synth.positions(32, 7)
    t = train.targets(32, 8)
    shard = pos.slice(rank * 16, rank * 16 + 16)
    st, _, g = oracle.t_grad(params, shard, t[rank * 16: rank * 16 + 16])
    assert st == 0
    grads = torch.from_numpy(g)
    w = train.allreduce_sum_(grads)  # the product's exchange step
    np.save(os.path.join(out_dir, f"g{rank}.npy"), grads.numpy() / w)
    dist.barrier()
    dist.destroy_process_group()


def test_data_parallel_exchange_equals_full_batch_gradient(params, tmp_path):
    import torch.multiprocessing as mp
    port = 29500 + os.getpid() % 1000
    mp.spawn(_dp_rank, args=(2, port, params, str(tmp_path)), nprocs=2, join=True)
    g0, g1 = np.load(tmp_path / "g0.npy"), np.load(tmp_path / "g1.npy")
    np.testing.assert_array_equal(g0, g1)  # every rank holds the same averaged gradient
    pos = synth.positions(32, 7)
    st, _, full = oracle.t_grad(params, pos, train.targets(32, 8))
    assert st == 0
    scale = np.abs(full).max()
    np.testing.assert_allclose(g0, full, rtol=1e-4, atol=1e-6 * scale)
