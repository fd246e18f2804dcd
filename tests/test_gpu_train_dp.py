"""Data-parallel HalfKA training step on two GPUs (skipped with fewer): two
NCCL ranks each stepping on half of a batch - the stack gradients all-reduced
beside the FT backward, the FT gradient either reduce-scattered with a
sharded Adam and an all-gather of the bf16 shadow, or all-reduced in row
chunks - end with bit-identical parameters, and their summed gradient
divided by the world size equals one rank's gradient of the whole batch
within the single-GPU parity tolerance."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
RTOL = 1e-4


def _batch():
    from chineseai_b200 import train
    from tests import _trainref
    params = train.init_params(3)
    pos, t, _ = _trainref.safe_batch(params, 4096, 31)
    if pos.n % 2:  # equal halves
        keep = np.ones(pos.n, bool)
        keep[-1] = False
        pos, t = _trainref.select(pos, keep), t[keep]
    return params, pos, t


def _half(pos, t, rank):
    from tests._trainref import select
    n = pos.n
    keep = np.zeros(n, bool)
    keep[rank * (n // 2):(rank + 1) * (n // 2)] = True
    return select(pos, keep), t[keep]


def _rank(rank, world, port, out, shard):
    import datetime

    import torch.distributed as dist
    from chineseai_b200 import train
    from chineseai_b200.quantized import as_device
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    params, pos, t = _batch()
    mine, tm = _half(pos, t, rank)
    tr = train.Trainer(params, rank, group=dist.group.WORLD, shard=shard, ft_chunks=1 if shard else 4)
    tr.step(as_device(mine.indices, dev), len(mine.indices), as_device(mine.offsets, dev), mine.n,
            torch.from_numpy(tm).to(dev))
    tr.gather_state()
    torch.cuda.synchronize()
    out[rank] = (tr.grads.cpu().numpy() / world, tr.params.cpu().numpy(), float(tr.flag.item()))
    dist.barrier()
    del tr
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shard", [True, False])
def test_two_rank_overlapped_step_equals_full_batch(shard):
    from chineseai_b200 import train
    from chineseai_b200.quantized import as_device
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29800 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port + int(shard), out, shard)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
        assert p.exitcode == 0
    g0, p0, f0 = out[0]
    g1, p1, f1 = out[1]
    assert f0 == 0.0 and f1 == 0.0
    np.testing.assert_array_equal(p0, p1)
    np.testing.assert_array_equal(g0, g1)
    # the halves' mean gradients, averaged, are the whole batch's
    params, pos, t = _batch()
    halves = [_half(pos, t, r) for r in range(2)]
    ref = train.Trainer(params, 0)
    dev = ref.device
    ref.forward_backward(as_device(pos.indices, dev), len(pos.indices), as_device(pos.offsets, dev), pos.n,
                         torch.from_numpy(t).to(dev))
    torch.cuda.synchronize()
    rg = ref.grads.cpu().numpy()
    gs, rs = train.split(g0), train.split(rg)
    for name, _ in train.LAYOUT:
        scale = np.abs(rs[name]).max()
        np.testing.assert_allclose(gs[name], rs[name], rtol=RTOL, atol=1e-5 * scale, err_msg=name)
    assert halves[0][0].n == halves[1][0].n
