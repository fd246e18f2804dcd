"""The torch-CPU restatement of the AZ training forward (oracle.az_train_ref)
checked piece by piece against the oracle's C twins of the reference's
custom ops (feature_pool, sparse_pool, fused_policy, sparse/tactical
lookups) on packed synthetic batches."""
import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import az, az_train
from oracle import az_train_ref
from tests._azutil import full_policy, trained_like


@pytest.fixture(scope="module")
def setup():
    w = az.AzWeights.random(32, 20260807)
    trained_like(w, 1)
    full_policy(w, 2)
    s = az_train.random_samples(24, 7)
    return w, az_train.pack_batch(s)


def test_reference_forward_pieces_match_c_twins(setup):
    w, b = setup
    t = [torch.tensor(x, dtype=torch.float64) for x in w.tensors()]
    value_logits, policy_logits = az_train_ref.forward(t, b)
    tens = w.tensors()
    # policy: fused + sparse + tactical through the C twins
    h = w.hidden
    ft = np.concatenate(tens[:5])
    st, pooled = oracle.feature_pool_fwd(ft, b.feature_items, h)
    assert st == 0
    board_pre = pooled.astype(np.float64) + tens[6]
    sh = np.maximum(board_pre + b.rule_context.astype(np.float64) @ tens[5], 0)
    hidden = sh / np.sqrt((sh * sh).mean(1, keepdims=True) + 1e-6)
    st, thr = oracle.sparse_pool_fwd(tens[10], b.value_threat_indices)
    assert st == 0
    act = np.clip(thr.astype(np.float64), 0, 1)
    pair = np.concatenate([act, act * act], 1)
    ctx = np.concatenate([hidden @ tens[15].T + pair @ tens[12].T, board_pre @ tens[17].T], 1).astype(np.float32)
    tables = np.concatenate([tens[0][:, :32].reshape(-1), tens[14], tens[13], tens[16].reshape(-1),
                             (tens[0].astype(np.float64) @ tens[17].T.astype(np.float64)).reshape(-1),
                             tens[18].reshape(-1)]).astype(np.float32)
    st, fused = oracle.policy_fused_fwd(tables, ctx, b.policy_items)
    assert st == 0
    st, sparse = oracle.policy_table_fwd(np.concatenate([tens[19], tens[20]]), b.policy_sparse_indices)
    assert st == 0
    st, tact = oracle.policy_table_fwd(np.concatenate([tens[21], [0.0]]).astype(np.float32),
                                       b.policy_tactical_indices)
    assert st == 0
    want = fused.astype(np.float64) + sparse + tact
    np.testing.assert_allclose(policy_logits.numpy(), want, rtol=1e-4, atol=1e-4)
    vh = np.maximum(hidden @ tens[7].T + tens[8], 0)
    vl = vh @ tens[9].T + pair @ tens[11].T
    np.testing.assert_allclose(value_logits.numpy(), vl, rtol=1e-5, atol=1e-5)


def test_reference_gradients_finite_and_loss_positive(setup):
    w, b = setup
    loss, grads = az_train_ref.gradients(w.tensors(), b)
    assert loss > 0 and all(np.isfinite(g).all() for g in grads)
    assert np.abs(grads[0]).max() > 0 and np.abs(grads[19]).max() > 0 and np.abs(grads[10]).max() > 0
