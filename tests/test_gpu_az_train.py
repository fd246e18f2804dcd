"""GPU checks of the AZ training step: the AdamW kernel equals the oracle's
restatement bit for bit; one step's loss and all 22 gradients match the
torch-CPU restatement of the reference forward (float64 autograd) within
1e-4 of each tensor's scale; the update is AdamW of those gradients; steps
are deterministic and a fixed batch overfits."""
import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import az, az_train
from chineseai_b200._lib import check, lib
from oracle import az_train_ref
from tests._azutil import full_policy, trained_like

pytestmark = pytest.mark.gpu
dev = torch.device("cuda", 0)


@pytest.mark.parametrize("n,offset", [(1000, 0), (1003, 1), (3, 0)])
def test_adamw_kernel_bit_exact(n, offset):
    rng = np.random.default_rng(n)
    p = rng.standard_normal(n + offset).astype(np.float32)
    m = (rng.standard_normal(n + offset) * 0.01).astype(np.float32)
    v = (rng.random(n + offset) * 1e-4).astype(np.float32)
    g = rng.standard_normal(n + offset).astype(np.float32)
    g[offset:offset + 3] = 0.0
    tp, tm, tv, tg = (torch.from_numpy(a.copy()).to(dev) for a in (p, m, v, g))
    for step in (1, 2, 7):
        check(lib().cnnue_adamw(tp.data_ptr() + 4 * offset, tm.data_ptr() + 4 * offset, tv.data_ptr() + 4 * offset,
                                tg.data_ptr() + 4 * offset, n, 1e-3, 0.9, 0.999, 1e-8, 1e-4, step, 0),
              "cnnue_adamw")
        pp, mm, vv = p[offset:].copy(), m[offset:].copy(), v[offset:].copy()
        oracle.adamw(pp, mm, vv, g[offset:], 1e-3, step=step)
        p[offset:], m[offset:], v[offset:] = pp, mm, vv
        torch.cuda.synchronize()
        np.testing.assert_array_equal(tp.cpu().numpy(), p)
        np.testing.assert_array_equal(tm.cpu().numpy(), m)
        np.testing.assert_array_equal(tv.cpu().numpy(), v)


def make(hidden, n, seed):
    w = az.AzWeights.random(hidden, 20260807 + seed)
    trained_like(w, seed)
    full_policy(w, seed + 1)
    return w, az_train.pack_batch(az_train.random_samples(n, seed + 2))


@pytest.mark.parametrize("hidden,n", [(32, 48), (128, 96)])
def test_step_gradients_match_reference(hidden, n):
    w, b = make(hidden, n, 3)
    tr = az_train.AzTrainer(w, lr=1e-3)
    bt = tr.to_device(b)
    tr.grad.zero_()
    loss, metrics = tr.loss(bt)
    loss.backward()
    grads = tr.gradients()
    ref_loss, ref_grads = az_train_ref.gradients(w.tensors(), b)
    assert abs(float(loss.detach()) - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss))
    for i, (g, r) in enumerate(zip(grads, ref_grads)):
        scale = max(np.abs(r).max(), 1e-12)
        err = np.abs(g.astype(np.float64) - r).max()
        assert err <= 1e-4 * scale + 1e-9, f"tensor {i} ({w.names[i]}): err {err} scale {scale}"
    # the update is AdamW of exactly these gradients
    p0 = [t.copy() for t in tr.tensors()]
    tr.step_count += 1
    check(lib().cnnue_adamw(tr.flat.data_ptr(), tr.m.data_ptr(), tr.v.data_ptr(), tr.grad.data_ptr(), tr.n_params,
                            tr.lr, 0.9, 0.999, 1e-8, 1e-4, tr.step_count, 0), "cnnue_adamw")
    after = tr.tensors()
    for i in (0, 10, 19, 21):
        p = p0[i].reshape(-1).copy()
        mm, vv = np.zeros_like(p), np.zeros_like(p)
        oracle.adamw(p, mm, vv, grads[i].reshape(-1), 1e-3, step=1)
        np.testing.assert_array_equal(after[i].reshape(-1), p)


def test_steps_deterministic_and_overfit():
    w, b = make(64, 64, 9)
    t1 = az_train.AzTrainer(w, lr=3e-3)
    t2 = az_train.AzTrainer(w, lr=3e-3)
    losses = []
    for _ in range(12):
        s1 = t1.step(b)
        t2.step(b)
        losses.append(s1.loss / s1.samples)
    for a, c in zip(t1.tensors(), t2.tensors()):
        np.testing.assert_array_equal(a, c)
    assert losses[-1] < 0.8 * losses[0], losses
    assert s1.samples == 64 and s1.phase[:, 0].sum() == 64


def test_copy_back_round_trip(tmp_path):
    w, b = make(32, 16, 4)
    tr = az_train.AzTrainer(w, lr=1e-3)
    tr.step(b)
    tr.copy_to(w)
    path = tmp_path / "w.safetensors"
    w.save(str(path))
    w2 = az.AzWeights.load(str(path))
    for a, c in zip(tr.tensors(), w2.tensors()):
        np.testing.assert_array_equal(a, c)


def test_bad_batch_raises_after_step():
    from chineseai_b200._lib import CnnueError
    w, b = make(32, 8, 5)
    b.policy_items[0, 0] = (3000 | 1 << 47)  # a move index past the 2086-move space
    tr = az_train.AzTrainer(w, lr=1e-3)
    with pytest.raises(CnnueError):
        tr.step(b)


def test_graph_steps_equal_eager_steps():
    """The captured step replays exactly what the eager step computes, step
    after step (device-side AdamW counter), on fixed-shape batches."""
    w, _ = make(64, 8, 12)
    s = az_train.random_samples(256, 13)
    batches = [az_train.pack_batch(s, np.arange(k * 64, (k + 1) * 64), caps=(40, 96, 96), fixed=True)
               for k in range(4)]
    eager = az_train.AzTrainer(w, lr=2e-3)
    graph = az_train.AzTrainer(w, lr=2e-3, graph=True)
    for k in range(6):
        b = batches[k % 4]
        se, sg = eager.step(b), graph.step(b)
        assert se.loss == sg.loss, (k, se.loss, sg.loss)
    assert graph._graph is not None
    for a, c in zip(eager.tensors(), graph.tensors()):
        np.testing.assert_array_equal(a, c)
    graph.set_learning_rate(1e-4)
    eager.set_learning_rate(1e-4)
    eager.step(batches[0])
    graph.step(batches[0])
    for a, c in zip(eager.tensors(), graph.tensors()):
        np.testing.assert_array_equal(a, c)


def test_gpu_index_expansion_matches_host_packer():
    s = az_train.random_samples(200, 21)
    full = az_train.pack_batch(s, caps=(40, 96, 96), fixed=True)
    comp = az_train.pack_batch(s, caps=(40, 96, 96), fixed=True, compact=True)
    w, _ = make(32, 4, 22)
    tr = az_train.AzTrainer(w)
    ex = tr.expand(tr.to_device(comp))
    np.testing.assert_array_equal(ex["policy_sparse_indices"].cpu().numpy(), full.policy_sparse_indices)
    np.testing.assert_array_equal(ex["policy_tactical_indices"].cpu().numpy(), full.policy_tactical_indices)
    np.testing.assert_array_equal(ex["policy_mask"].cpu().numpy(), full.policy_mask)


def test_compact_batches_train_identically():
    s = az_train.random_samples(128, 23)
    rows = [np.arange(k * 64, (k + 1) * 64) for k in range(2)]
    full = [az_train.pack_batch(s, r, caps=(40, 96, 96), fixed=True) for r in rows]
    comp = [az_train.pack_batch(s, r, caps=(40, 96, 96), fixed=True, compact=True) for r in rows]
    w, _ = make(32, 4, 24)
    a = az_train.AzTrainer(w, lr=2e-3)
    b = az_train.AzTrainer(w, lr=2e-3, graph=True)
    for k in range(4):
        sa, sb = a.step(full[k % 2]), b.step(comp[k % 2])
        assert sa.loss == sb.loss
    for x, y in zip(a.tensors(), b.tensors()):
        np.testing.assert_array_equal(x, y)
