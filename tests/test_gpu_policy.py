"""GPU parity of the policy-head training ops (fused_policy, sparse_policy,
tactical_policy), forward and the atomic-free backward, against the oracle:
the reference test's fixture (src/az/fused_policy.rs:536-572) bit for bit,
random batches bit for bit wherever a table entry takes at most 256
contributions (elsewhere within the float32 bound of the summation), and
run-to-run determinism."""
import os

import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import policy
from chineseai_b200._lib import CnnueError
from tests.golden.make_golden import policy_fixture
from tests.test_oracle_policy import random_policy

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
dev = torch.device("cuda", 0)


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_reference_fixture_forward_and_gradient():
    g = np.load(GOLDEN)
    tab, ctx, items = policy_fixture()
    tt = t(tab).requires_grad_()
    ct = t(ctx).requires_grad_()
    out = policy.fused_policy(tt, ct, t(items))
    np.testing.assert_array_equal(out.detach().cpu().numpy(), g["policy_fwd"])
    out.sum().backward()
    full = np.zeros(policy.TABLE_LEN, np.float32)
    full[g["policy_grad_idx"]] = g["policy_grad_val"]
    np.testing.assert_array_equal(tt.grad.cpu().numpy(), full)
    np.testing.assert_array_equal(ct.grad.cpu().numpy(), g["policy_grad_context"])


def contribution_bound(tab, ctx, items, grad):
    """Per-entry bound on |float32 sum - exact sum| for the consequence
    weights (every move item adds to all 32): n * eps * sum |terms|."""
    bound = np.zeros(32)
    count = 0
    for b in range(items.shape[0]):
        for m in range(items.shape[1]):
            p = int(items[b, m]) & (2**64 - 1)
            if not ((p >> 47) & 1 and (p >> 45) & 1):
                continue
            fr, to, cp = (p >> 12) & 0x7ff, (p >> 23) & 0x7ff, (p >> 34) & 0x7ff
            d = tab[to * 32:to * 32 + 32].astype(np.float64) - tab[fr * 32:fr * 32 + 32]
            if (p >> 46) & 1:
                d -= tab[cp * 32:cp * 32 + 32]
            bound += np.abs(grad[b, m] * d)
            count += 1
    return count, bound * count * 2.0**-23 + 1e-30


@pytest.mark.parametrize("batch,moves,seed", [(1, 1, 1), (7, 13, 2), (64, 48, 3), (300, 90, 4)])
def test_random_batches(batch, moves, seed):
    tab, ctx, items = random_policy(batch, moves, seed)
    grad = np.random.default_rng(seed + 100).standard_normal(items.shape).astype(np.float32)
    st, ref = oracle.policy_fused_fwd(tab, ctx, items)
    assert st == 0
    out = policy.fused_policy_forward(t(tab), t(ctx), t(items)).cpu().numpy()
    np.testing.assert_array_equal(out, ref)
    st, rgt, rgc = oracle.policy_fused_bwd(tab, ctx, items, grad)
    assert st == 0
    gt, gc = policy.fused_policy_backward(t(tab), t(ctx), t(items), t(grad))
    gt, gc = gt.cpu().numpy(), gc.cpu().numpy()
    np.testing.assert_array_equal(gc, rgc)
    count, bound = contribution_bound(tab, ctx, items, grad)
    cons = slice(40320, 40352)
    if items.size <= 256:  # the consequence weights sum in ordered chunks of 256 items
        np.testing.assert_array_equal(gt, rgt)
    else:
        keep = np.ones(len(gt), bool)
        keep[cons] = False
        np.testing.assert_array_equal(gt[keep], rgt[keep])
        assert np.all(np.abs(gt[cons].astype(np.float64) - rgt[cons]) <= 2 * bound)
    gt2, gc2 = policy.fused_policy_backward(t(tab), t(ctx), t(items), t(grad))
    np.testing.assert_array_equal(gt2.cpu().numpy(), gt)  # deterministic
    np.testing.assert_array_equal(gc2.cpu().numpy(), gc)


def test_empty_batch():
    tab = np.zeros(policy.TABLE_LEN, np.float32)
    out = policy.fused_policy_forward(t(tab), t(np.zeros((0, 48), np.float32)), t(np.zeros((0, 5), np.int64)))
    assert out.shape == (0, 5)
    gt, gc = policy.fused_policy_backward(t(tab), t(np.zeros((0, 48), np.float32)), t(np.zeros((0, 5), np.int64)),
                                          t(np.zeros((0, 5), np.float32)))
    assert gc.shape == (0, 48) and not gt.any()


def test_bad_item_raises():
    tab, ctx, items = policy_fixture()
    items = items.copy()
    items[0, 1] = policy.pack_policy_item(5, 1300, 2, 0, True, False)  # from past the 1260 features
    with pytest.raises(CnnueError):
        policy.fused_policy(t(tab), t(ctx), t(items))
    with pytest.raises(CnnueError):
        policy.fused_policy_backward(t(tab), t(ctx), t(items), t(np.ones((2, 3), np.float32)))


def test_shape_errors():
    tab, ctx, items = policy_fixture()
    with pytest.raises(ValueError):
        policy.fused_policy(t(tab[:-1]), t(ctx), t(items))
    with pytest.raises(ValueError):
        policy.sparse_policy(t(tab), t(np.zeros((2, 3, 2), np.int64)))
    with pytest.raises(ValueError):
        policy.tactical_policy(t(tab), t(np.zeros((2, 3, 7), np.int64)))


@pytest.mark.parametrize("terms,table_len,batch,moves", [(7, 2396815, 256, 60), (2, 41, 64, 40), (7, 5000, 3, 4)])
def test_table_ops(terms, table_len, batch, moves):
    rng = np.random.default_rng(terms * 1000 + batch)
    table = rng.standard_normal(table_len).astype(np.float32)
    idx = rng.integers(0, table_len, size=(batch, moves, terms)).astype(np.int64)
    st, ref = oracle.policy_table_fwd(table, idx)
    assert st == 0
    tt = t(table).requires_grad_()
    fn = policy.sparse_policy if terms == 7 else policy.tactical_policy
    out = fn(tt, t(idx))
    np.testing.assert_array_equal(out.detach().cpu().numpy(), ref)
    g = rng.standard_normal((batch, moves)).astype(np.float32)
    out.backward(t(g))
    st, rgrad = oracle.policy_table_bwd(idx, g, table_len)
    assert st == 0
    grad = tt.grad.cpu().numpy()
    counts = np.bincount(idx.reshape(-1), minlength=table_len)
    exact = counts <= 256
    np.testing.assert_array_equal(grad[exact], rgrad[exact])
    if not exact.all():  # a small table: long runs are summed in ordered units of 256
        hits = idx.reshape(-1)
        vals = np.repeat(g.reshape(-1), terms).astype(np.float64)
        mag = np.zeros(table_len)
        np.add.at(mag, hits, np.abs(vals))
        err = np.abs(grad[~exact].astype(np.float64) - rgrad[~exact])
        assert np.all(err <= 2 * counts[~exact] * 2.0**-23 * mag[~exact])
    assert np.array_equal(policy.table_backward(t(idx), t(g), table_len).cpu().numpy(), grad)


def test_table_bad_index_raises():
    table = t(np.ones(10, np.float32))
    with pytest.raises(CnnueError):
        policy.tactical_policy(table, t(np.array([[[1, 12]]], np.int64)))
    with pytest.raises(CnnueError):
        policy.table_backward(t(np.array([[[1, -1]]], np.int64)), t(np.ones((1, 1), np.float32)), 10)
