"""GPU checks of the native AZ-NNUE training step (cnnue_azt_step): the loss,
the 30 statistics and all 22 gradients against the float64 torch-CPU
restatement of the reference forward (oracle/az_train_ref.py) within 1e-4 of
each tensor's scale; padded fixed-width batches (whose padded moves are not
enumerated) and compact batches give the same bits as full ones; the step is
deterministic; bad indices raise after the step."""
import numpy as np
import pytest
import torch

from chineseai_b200 import az, az_train
from chineseai_b200._lib import CnnueError
from oracle import az_train_ref
from tests._azutil import full_policy, trained_like

pytestmark = pytest.mark.gpu


def make(hidden, seed):
    w = az.AzWeights.random(hidden, 20260807 + seed)
    trained_like(w, seed)
    full_policy(w, seed + 1)
    return w


def native_grads(tr, b, vw=1.0, pw=1.0):
    m = tr.native_loss(tr.to_device(b), vw, pw).cpu().numpy()
    return m, tr.gradients()


def check_against_reference(w, b, tr, vw=1.0, pw=1.0):
    m, grads = native_grads(tr, b, vw, pw)
    assert m[30] == 0.0, f"status word {m[30]}"
    ref_loss, ref_grads = az_train_ref.gradients(w.tensors(), b, vw, pw)
    loss = m[0] / b.batch_size
    assert abs(loss - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss)), (loss, ref_loss)
    for i, (g, r) in enumerate(zip(grads, ref_grads)):
        scale = max(np.abs(r).max(), 1e-12)
        err = np.abs(g.astype(np.float64) - r).max()
        assert err <= 1e-4 * scale + 1e-9, f"tensor {i} ({w.names[i]}): err {err} scale {scale}"
    return m


@pytest.mark.parametrize("hidden,n", [(32, 48), (64, 33), (128, 96), (256, 20)])
def test_native_gradients_match_reference(hidden, n):
    w = make(hidden, 3)
    b = az_train.pack_batch(az_train.random_samples(n, 5))
    tr = az_train.AzTrainer(w, lr=1e-3)
    assert tr.native
    check_against_reference(w, b, tr)
    tr.close()


def test_native_padded_batch_and_loss_weights():
    """Fixed widths leave padded moves, threats and feature items (dropped
    before the sort); unequal value / policy weights scale each term."""
    w = make(128, 7)
    s = az_train.random_samples(80, 8)
    b = az_train.pack_batch(s, caps=(40, 96, 96), fixed=True)
    tr = az_train.AzTrainer(w, lr=1e-3)
    check_against_reference(w, b, tr, vw=0.5, pw=2.0)
    tr.close()


def test_native_statistics_match_torch_path():
    w = make(64, 11)
    b = az_train.pack_batch(az_train.random_samples(64, 12))
    nat = az_train.AzTrainer(w, lr=1e-3)
    ref = az_train.AzTrainer(w, lr=1e-3, native=False)
    m, g_nat = native_grads(nat, b)
    bt = ref.to_device(b)
    ref.grad.zero_()
    loss, metrics = ref.loss(bt)
    loss.backward()
    mt = metrics.cpu().numpy()
    np.testing.assert_allclose(m[:30], mt, rtol=2e-5, atol=2e-5)
    for a, c in zip(g_nat, ref.gradients()):
        scale = max(np.abs(c).max(), 1e-12)
        assert np.abs(a - c).max() <= 1e-4 * scale + 1e-9
    nat.close()


def test_native_deterministic_and_compact_equal_full():
    w = make(128, 13)
    s = az_train.random_samples(128, 14)
    full = az_train.pack_batch(s, caps=(40, 96, 96), fixed=True)
    comp = az_train.pack_batch(s, caps=(40, 96, 96), fixed=True, compact=True)
    tr = az_train.AzTrainer(w, lr=1e-3)
    m1, g1 = native_grads(tr, full)
    m2, g2 = native_grads(tr, full)
    m3, g3 = native_grads(tr, comp)
    np.testing.assert_array_equal(m1, m2)
    np.testing.assert_array_equal(m1, m3)
    for a, b_, c in zip(g1, g2, g3):
        np.testing.assert_array_equal(a, b_)
        np.testing.assert_array_equal(a, c)
    tr.close()


def test_native_graph_steps_equal_eager_steps():
    w = make(128, 15)
    s = az_train.random_samples(256, 16)
    batches = [az_train.pack_batch(s, np.arange(k * 64, (k + 1) * 64), caps=(40, 96, 96), fixed=True, compact=True)
               for k in range(4)]
    eager = az_train.AzTrainer(w, lr=2e-3)
    graph = az_train.AzTrainer(w, lr=2e-3, graph=True)
    for k in range(6):
        se, sg = eager.step(batches[k % 4]), graph.step(batches[k % 4])
        assert se.loss == sg.loss, (k, se.loss, sg.loss)
    assert graph._graph is not None
    for a, c in zip(eager.tensors(), graph.tensors()):
        np.testing.assert_array_equal(a, c)
    eager.close()
    graph.close()


@pytest.mark.parametrize("field,value", [("policy_items", 3000 | 1 << 47), ("value_threat_indices", 60000),
                                         ("feature_items", 2047), ("policy_sparse_indices", 1 << 40)])
def test_native_bad_index_raises_after_step(field, value):
    w = make(32, 17)
    b = az_train.pack_batch(az_train.random_samples(8, 18))
    arr = getattr(b, field)
    arr.reshape(-1)[0] = value
    tr = az_train.AzTrainer(w, lr=1e-3)
    with pytest.raises(CnnueError):
        tr.step(b)
    # the next good batch is clean
    good = az_train.pack_batch(az_train.random_samples(8, 19))
    tr.step(good)
    tr.close()
