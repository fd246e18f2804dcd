"""GPU parity of the training step (cnnue_t_*) against the oracle: loss and
every gradient within rtol 1e-4 (atol 1e-5 of each tensor's largest entry),
Adam within 1e-6, the bf16 shadow exactly, run-to-run determinism, and the
data errors.  Parity batches leave out the few positions whose hidden
pre-activations sit within 1e-5 of a clamp boundary (tests/_trainref.py):
there two correct summation orders may pick different masks."""
import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import synth, train
from chineseai_b200._lib import CnnueError
from chineseai_b200.quantized import as_device
from tests import _trainref

pytestmark = pytest.mark.gpu
RTOL = 1e-4


@pytest.fixture(scope="module")
def params():
    return train.init_params(3)


def run_fb(tr, pos, t):
    idx, off = as_device(pos.indices, tr.device), as_device(pos.offsets, tr.device)
    tt = torch.from_numpy(t).to(tr.device)
    tr.forward_backward(idx, len(pos.indices), off, pos.n, tt)
    assert tr.status() == 0
    torch.cuda.synchronize()
    return float(tr.loss.item()), tr.grads.cpu().numpy().copy()


@pytest.mark.parametrize("n,seed", [(64, 11), (1500, 12)])
def test_forward_backward_matches_oracle(params, n, seed):
    tr = train.Trainer(params, 0)
    pos, t, _ = _trainref.safe_batch(params, n, seed)
    loss, g = run_fb(tr, pos, t)
    st, ref_loss, ref_g = oracle.t_grad(params, pos, t)
    assert st == 0
    assert abs(loss - ref_loss) <= RTOL * abs(ref_loss)
    gs, rs = train.split(g), train.split(ref_g)
    for name, _ in train.LAYOUT:
        scale = np.abs(rs[name]).max()
        np.testing.assert_allclose(gs[name], rs[name], rtol=RTOL, atol=1e-5 * scale, err_msg=name)


def test_shadow_and_adam_match_oracle(params):
    tr = train.Trainer(params, 0)
    shadow = tr.shadow.cpu().numpy().view(np.uint16)
    ref_shadow = oracle.bf16_round(params[: train.SHADOW]).view(np.uint32) >> 16
    np.testing.assert_array_equal(shadow, ref_shadow.astype(np.uint16))
    pos = synth.positions(128, 13)
    t = train.targets(128, 14)
    _, g = run_fb(tr, pos, t)
    tr.apply_adam(0.5)
    torch.cuda.synchronize()
    w, m, v = params.copy(), np.zeros_like(params), np.zeros_like(params)
    oracle.adam(w, m, v, g, 0.5, 1e-3, 0.9, 0.999, 1e-8, 1)
    np.testing.assert_allclose(tr.params.cpu().numpy(), w, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(tr.m.cpu().numpy(), m, rtol=1e-6, atol=1e-12)
    np.testing.assert_allclose(tr.v.cpu().numpy(), v, rtol=1e-5, atol=1e-18)
    shadow = tr.shadow.cpu().numpy().view(np.uint16)
    ref_shadow = (oracle.bf16_round(tr.params.cpu().numpy()[: train.SHADOW]).view(np.uint32) >> 16)
    np.testing.assert_array_equal(shadow, ref_shadow.astype(np.uint16))


def test_gradients_are_deterministic(params):
    tr = train.Trainer(params, 0)
    pos = synth.positions(16384, 15)
    t = train.targets(16384, 16)
    l1, g1 = run_fb(tr, pos, t)
    l2, g2 = run_fb(tr, pos, t)
    assert l1 == l2
    np.testing.assert_array_equal(g1, g2)
    assert np.isfinite(g1).all()


def test_full_batch_gradient_within_tolerance(params):
    tr = train.Trainer(params, 0)
    pos, t, dropped = _trainref.safe_batch(params, 16384, 17)
    assert dropped < 100
    loss, g = run_fb(tr, pos, t)
    st, ref_loss, ref_g = oracle.t_grad(params, pos, t)
    assert st == 0
    assert abs(loss - ref_loss) <= RTOL * abs(ref_loss)
    gs, rs = train.split(g), train.split(ref_g)
    for name, _ in train.LAYOUT:
        scale = np.abs(rs[name]).max()
        np.testing.assert_allclose(gs[name], rs[name], rtol=RTOL, atol=1e-5 * scale, err_msg=name)


def test_training_reduces_loss(params):
    tr = train.Trainer(params, 0, train.AdamConfig(lr=1e-2))
    pos = synth.positions(2048, 19)
    t = train.targets(2048, 20)
    losses = [tr.step_positions(pos, t) for _ in range(20)]
    assert losses[-1] < losses[0]


def test_bad_index_is_reported(params):
    tr = train.Trainer(params, 0)
    pos = synth.Positions(np.array([1, 11340, 5, 6], np.uint16), np.array([0, 2, 4], np.uint32))
    with pytest.raises(CnnueError) as e:
        tr.step_positions(pos, np.zeros(1, np.float32))
    assert e.value.status == 2
