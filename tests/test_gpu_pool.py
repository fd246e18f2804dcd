"""GPU parity of the AZ-NNUE feature pool and plain pool, forward and the
atomic-free backward, on the reference's own test fixtures
(src/az/fused_feature_pool.rs:611-686) and on random batches."""
import os

import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import pool
from tests.golden.make_golden import pool_fixture, sparse_fixture

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
dev = torch.device("cuda", 0)
PAD_ITEM = 0xFFFFFFFF


def t(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(dev)


def test_reference_fixture_forward_and_gradient():
    g = np.load(GOLDEN)
    tables, items = pool_fixture()
    out = pool.feature_pool(t(tables), t(items)).cpu().numpy()
    np.testing.assert_array_equal(out, g["pool_fwd"])
    grad = pool.feature_pool_backward(t(items), t(np.ones((2, 7), np.float32))).cpu().numpy()
    np.testing.assert_array_equal(grad, g["pool_bwd"])


def test_sparse_reference_fixture():
    g = np.load(GOLDEN)
    table, items = sparse_fixture()
    out = pool.sparse_pool(t(table), t(items)).cpu().numpy()
    np.testing.assert_array_equal(out, g["sparse_fwd"])
    grad = pool.sparse_pool_backward(t(items), t(np.ones((2, 7), np.float32)), 11).cpu().numpy()
    np.testing.assert_array_equal(grad, g["sparse_bwd"])


def random_items(batch, item_count, seed):
    rng = np.random.default_rng(seed)
    feat = rng.integers(0, 1260, size=(batch, item_count))
    us = rng.integers(0, 9, size=(batch, 1))
    them = rng.integers(0, 9, size=(batch, 1))
    items = (feat | (us << 11) | (them << 15)).astype(np.uint32)
    n_valid = rng.integers(0, item_count + 1, size=batch)
    items[np.arange(item_count)[None, :] >= n_valid[:, None]] = 0xFFFFFFFF
    return items


@pytest.mark.parametrize("batch,items_per,hidden", [(3, 5, 7), (64, 32, 128), (300, 40, 96)])
def test_forward_bit_exact(batch, items_per, hidden):
    rng = np.random.default_rng(batch)
    tables = rng.standard_normal((1545, hidden)).astype(np.float32)
    items = random_items(batch, items_per, batch + 1)
    out = pool.feature_pool(t(tables), t(items)).cpu().numpy()
    st, ref = oracle.feature_pool_fwd(tables, items, hidden)
    assert st == 0
    np.testing.assert_array_equal(out, ref)


def test_backward_small_is_bit_exact():
    # every row has <= 256 contributions -> the reference CPU order exactly
    items = random_items(20, 8, 5)
    grad_out = np.random.default_rng(6).standard_normal((20, 16)).astype(np.float32)
    grad = pool.feature_pool_backward(t(items), t(grad_out)).cpu().numpy()
    st, ref = oracle.feature_pool_bwd(items, grad_out, 16)
    assert st == 0
    np.testing.assert_array_equal(grad, ref)


@pytest.mark.parametrize("batch,hidden", [(1024, 128), (700, 7)])
def test_backward_large_within_tolerance_and_deterministic(batch, hidden):
    items = random_items(batch, 32, 9)
    grad_out = np.random.default_rng(10).standard_normal((batch, hidden)).astype(np.float32)
    g1 = pool.feature_pool_backward(t(items), t(grad_out)).cpu().numpy()
    g2 = pool.feature_pool_backward(t(items), t(grad_out)).cpu().numpy()
    np.testing.assert_array_equal(g1, g2)
    st, ref = oracle.feature_pool_bwd(items, grad_out, hidden)
    assert st == 0
    scale = np.abs(ref).max()
    np.testing.assert_allclose(g1, ref, rtol=1e-4, atol=1e-5 * scale)


def test_bad_item_is_flagged():
    from chineseai_b200._lib import CnnueError
    tables = np.zeros((1545, 4), np.float32)
    items = np.array([[0 | (15 << 15)]], np.uint32)
    with pytest.raises(CnnueError):
        pool.feature_pool(t(tables), t(items))


@pytest.mark.parametrize("batch,item_count,hidden,seed", [(5, 9, 64, 1), (512, 48, 64, 2), (128, 30, 128, 3)])
def test_threat_table_backward(batch, item_count, hidden, seed):
    """The 57,702-row threat table (past the shared-memory histogram): bit
    exact wherever a row takes at most 256 contributions, deterministic."""
    rows = 57702
    rng = np.random.default_rng(seed)
    items = rng.integers(0, rows, size=(batch, item_count)).astype(np.uint32)
    items[:, -3:] = PAD_ITEM
    items[0, :5] = 4242  # a row hit repeatedly inside one batch row
    if batch >= 512:
        items[:, 0] = 7  # a row with `batch` (> 256) contributions
    grad_out = rng.standard_normal((batch, hidden)).astype(np.float32)
    table = rng.standard_normal((rows, hidden)).astype(np.float32)
    st, ref_fwd = oracle.sparse_pool_fwd(table, items)
    assert st == 0
    np.testing.assert_array_equal(pool.sparse_pool(t(table), t(items)).cpu().numpy(), ref_fwd)
    g1 = pool.sparse_pool_backward(t(items), t(grad_out), rows).cpu().numpy()
    g2 = pool.sparse_pool_backward(t(items), t(grad_out), rows).cpu().numpy()
    np.testing.assert_array_equal(g1, g2)
    st, ref = oracle.sparse_pool_bwd(items, grad_out, rows)
    assert st == 0
    counts = np.bincount(items[items != PAD_ITEM].astype(np.int64), minlength=rows)
    exact = counts <= 256
    np.testing.assert_array_equal(g1[exact], ref[exact])
    if not exact.all():
        mag = np.zeros((rows, hidden))
        valid = items != PAD_ITEM
        np.add.at(mag, items[valid].astype(np.int64), np.abs(np.repeat(grad_out, item_count, 0)[valid.reshape(-1)]))
        err = np.abs(g1[~exact].astype(np.float64) - ref[~exact])
        assert np.all(err <= 2 * counts[~exact, None] * 2.0**-23 * mag[~exact])


def test_threat_table_backward_bad_row_flagged():
    from chineseai_b200._lib import CnnueError
    items = np.array([[3, 57702]], np.uint32)
    with pytest.raises(CnnueError):
        pool.sparse_pool_backward(t(items), t(np.ones((1, 64), np.float32)), 57702)
