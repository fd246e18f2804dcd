"""CPU tests of the oracle: agreement with an independent numpy restatement,
the golden fixtures, the reference's own feature-pool fixtures, and edge
cases.  No GPU needed."""
import hashlib
import os

import numpy as np
import pytest

import oracle
from chineseai_b200 import synth
from tests import _npref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_generators_match_golden_hashes(golden, qweights, fweights):
    for f in qweights.FIELDS:
        assert sha(getattr(qweights, f)) == str(golden[f"qw_sha_{f}"]), f
    for f in fweights.FIELDS:
        assert sha(getattr(fweights, f)) == str(golden[f"fw_sha_{f}"]), f
    pos = synth.positions(32, 1)
    np.testing.assert_array_equal(pos.indices, golden["q_idx"])
    np.testing.assert_array_equal(pos.offsets, golden["q_off"])
    big = synth.positions(65536, 1)
    assert sha(big.indices) == str(golden["q_big_idx_sha"])
    assert sha(big.offsets) == str(golden["q_big_off_sha"])


def test_position_generator_shape():
    pos = synth.positions(2000, 1)
    c = pos.counts()
    assert c.min() >= 2 and c.max() <= 32
    assert abs(c.mean() - 17.0) < 0.5
    for p in range(50):
        for s in range(2):
            seg = pos.indices[pos.offsets[2 * p + s]: pos.offsets[2 * p + s + 1]]
            assert np.all(np.diff(seg.astype(np.int64)) > 0)  # unique, sorted
            assert seg.max() < 11340


def test_q_oracle_matches_numpy_and_golden(golden, qweights):
    pos = synth.Positions(golden["q_idx"], golden["q_off"])
    st, scores, acc = oracle.q_forward(qweights, pos, with_acc=True)
    assert st == 0
    ref_scores, ref_acc = _npref.q_forward(qweights, pos)
    np.testing.assert_array_equal(acc, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)
    np.testing.assert_array_equal(scores, golden["q_scores"])
    assert sha(acc) == str(golden["q_acc_sha"])


def test_q_oracle_matches_numpy_random_batch(qweights):
    pos = synth.positions(300, 7)
    st, scores, acc = oracle.q_forward(qweights, pos, with_acc=True)
    ref_scores, ref_acc = _npref.q_forward(qweights, pos)
    assert st == 0
    np.testing.assert_array_equal(acc, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)


def test_q_oracle_wraparound_is_exercised(qweights):
    # With FT rows uniform in [-127,127] and up to 32 rows, sums stay inside
    # int16; force wraparound with a repeated index list.
    idx = np.full(600, 5, np.uint16)
    pos = synth.Positions(idx, np.array([0, 300, 600], np.uint32))
    st, scores, acc = oracle.q_forward(qweights, pos, with_acc=True)
    ref_scores, ref_acc = _npref.q_forward(qweights, pos)
    assert st == 0
    wide = qweights.ft_bias.astype(np.int64) + 300 * qweights.ft_weight[5].astype(np.int64)
    assert np.any(np.abs(wide) > 32767)
    np.testing.assert_array_equal(acc, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)


def test_q_oracle_edge_cases(qweights):
    # empty lists (count 0 -> bucket 0), a single position, long lists -> bucket 15
    idx = np.arange(40, dtype=np.uint16)
    pos = synth.Positions(idx, np.array([0, 0, 0, 40, 40], np.uint32))
    st, scores, acc = oracle.q_forward(qweights, pos, with_acc=True)
    ref_scores, ref_acc = _npref.q_forward(qweights, pos)
    assert st == 0
    np.testing.assert_array_equal(scores, ref_scores)
    np.testing.assert_array_equal(acc[0, 0], qweights.ft_bias)
    assert oracle.q_bucket(0) == 0 and oracle.q_bucket(1) == 0 and oracle.q_bucket(2) == 0
    assert oracle.q_bucket(3) == 1 and oracle.q_bucket(32) == 15 and oracle.q_bucket(40) == 15
    # bad index -> status 2; bad offsets -> status 3
    bad = synth.Positions(np.array([11340, 1], np.uint16), np.array([0, 1, 2], np.uint32))
    assert oracle.q_forward(qweights, bad)[0] == 2
    badoff = synth.Positions(np.array([1, 2], np.uint16), np.array([0, 2, 1], np.uint32))
    assert oracle.q_forward(qweights, badoff)[0] == 3


def test_q_oracle_multithread_equals_single(qweights):
    pos = synth.positions(1000, 3)
    st1, s1, _ = oracle.q_forward(qweights, pos)
    st2, s2 = oracle.q_forward_mt(qweights, pos, 4)
    assert st1 == st2 == 0
    np.testing.assert_array_equal(s1, s2)


def test_q_update_oracle(golden, qweights):
    ub = synth.UpdateBatch(golden["u_parent"], golden["u_flags"], golden["u_rem"], golden["u_rem_offsets"],
                           golden["u_add"], golden["u_add_offsets"], golden["u_count0"])
    st, child, scores = oracle.q_update(qweights, ub)
    assert st == 0
    ref_child, ref_scores = _npref.q_update(qweights, ub)
    np.testing.assert_array_equal(child, ref_child)
    np.testing.assert_array_equal(scores, ref_scores)
    np.testing.assert_array_equal(scores, golden["u_scores"])
    assert sha(child) == str(golden["u_child_sha"])
    fresh = synth.update_batch(32, 1)
    np.testing.assert_array_equal(fresh.parent, ub.parent)
    np.testing.assert_array_equal(fresh.add, ub.add)


def test_q_update_is_consistent_with_forward(qweights):
    # parent = forward accumulator of a position; removing/adding indices must
    # equal the forward of the edited lists (wraparound is a group).
    pos = synth.positions(20, 11)
    _, _, parent_acc = oracle.q_forward(qweights, pos, with_acc=True)
    rng = np.random.default_rng(0)
    new_idx, new_off, rem, rem_off, add, add_off, c0 = [], [0], [], [0], [], [0], []
    for p in range(pos.n):
        for s in range(2):
            seg = list(pos.indices[pos.offsets[2 * p + s]: pos.offsets[2 * p + s + 1]])
            r = seg[0]
            a = int(rng.integers(0, 11340))
            while a in seg:
                a = int(rng.integers(0, 11340))
            seg2 = sorted([x for x in seg if x != r] + [a])
            new_idx += seg2
            new_off.append(len(new_idx))
            rem.append(r)
            rem_off.append(len(rem))
            add.append(a)
            add_off.append(len(add))
            if s == 0:
                c0.append(len(seg2))
    child_pos = synth.Positions(np.array(new_idx, np.uint16), np.array(new_off, np.uint32))
    _, ref_scores, ref_acc = oracle.q_forward(qweights, child_pos, with_acc=True)
    ub = synth.UpdateBatch(parent_acc, np.zeros(2 * pos.n, np.uint8), np.array(rem, np.uint16),
                           np.array(rem_off, np.uint32), np.array(add, np.uint16), np.array(add_off, np.uint32),
                           np.array(c0, np.uint8))
    st, child, scores = oracle.q_update(qweights, ub)
    assert st == 0
    np.testing.assert_array_equal(child, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)


def test_f_oracle(golden, fweights):
    pos = synth.Positions(golden["q_idx"], golden["q_off"])
    st, out, acc = oracle.f_forward(fweights, pos, with_acc=True)
    assert st == 0
    np.testing.assert_array_equal(out, golden["f_out"])
    ref = _npref.f_forward(fweights, pos)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-6)


def test_f_oracle_ft_sums_follow_the_scalar_order(fweights):
    """The fp32 FT sums are bias first, then every row in index order, one
    float32 add each: the order the GPU kernel keeps bit for bit."""
    pos = synth.positions(64, 9)
    st, _, acc = oracle.f_forward(fweights, pos, with_acc=True)
    assert st == 0
    acc = np.asarray(acc, np.float32).reshape(pos.n, 2, 256)
    ft = np.asarray(fweights.ft_weight, np.float32)
    for q in range(pos.n):
        for p in range(2):
            s = np.asarray(fweights.ft_bias, np.float32).copy()
            for f in pos.indices[pos.offsets[2 * q + p]:pos.offsets[2 * q + p + 1]]:
                s = (s + ft[int(f)]).astype(np.float32)
            np.testing.assert_array_equal(acc[q, p], s)


def test_feature_pool_oracle_on_reference_fixture(golden):
    from tests.golden.make_golden import pool_fixture
    tables, items = pool_fixture()
    np.testing.assert_array_equal(items, golden["pool_items"])
    st, out = oracle.feature_pool_fwd(tables, items, 7)
    assert st == 0
    np.testing.assert_array_equal(out, _npref.feature_pool_fwd(tables, items))
    np.testing.assert_array_equal(out, golden["pool_fwd"])
    # The reference test differentiates sum_all(): grad_out = 1.
    st, grad = oracle.feature_pool_bwd(items, np.ones((2, 7), np.float32), 7)
    assert st == 0
    np.testing.assert_array_equal(grad, _npref.feature_pool_bwd(items, np.ones((2, 7), np.float32)))
    np.testing.assert_array_equal(grad, golden["pool_bwd"])
    # Item (95, 3, 4) appears twice: its feature row gets gradient 2.
    assert np.all(grad[95] == 2.0) and np.all(grad[0] == 1.0) and np.all(grad[1259] == 1.0)
    # float64 cross-check of the forward within the reference test's 2e-5
    t64 = tables.astype(np.float64)
    exp0 = sum(t64[r] for r in _npref.pool_item_rows(items[0, 0]) + _npref.pool_item_rows(items[0, 1]))
    np.testing.assert_allclose(out[0], exp0, atol=2e-5)


def test_sparse_pool_oracle_on_reference_fixture(golden):
    from tests.golden.make_golden import sparse_fixture
    table, items = sparse_fixture()
    st, out = oracle.sparse_pool_fwd(table, items)
    assert st == 0
    t64 = table.astype(np.float64)
    np.testing.assert_allclose(out[0], t64[1] + t64[4] + t64[1], atol=2e-5)
    np.testing.assert_allclose(out[1], t64[10] + t64[3] + t64[3], atol=2e-5)
    np.testing.assert_array_equal(out, golden["sparse_fwd"])
    st, grad = oracle.sparse_pool_bwd(items, np.ones((2, 7), np.float32), 11)
    counts = np.bincount(items[items != 0xFFFFFFFF].astype(np.int64), minlength=11)
    np.testing.assert_array_equal(grad, np.repeat(counts[:, None], 7, 1).astype(np.float32))
    np.testing.assert_array_equal(grad, golden["sparse_bwd"])


def test_feature_pool_oracle_flags_rows_past_table():
    tables = np.zeros((1545, 4), np.float32)
    items = np.array([[0 | (15 << 15)]], np.uint32)  # them bucket 15 -> row past 1545
    assert oracle.feature_pool_fwd(tables, items, 4)[0] == 2


def test_cpu_baseline_avx2_path_matches_scalar_oracle():
    """The timed CPU baseline (oracle_q_forward_mt: hand-written AVX2 row adds,
    pack and L1 when built for AVX2) is bit-identical to the scalar oracle,
    including int16 wraparound and empty lists."""
    import oracle
    from chineseai_b200 import synth
    w = synth.quantized_weights(2)
    cases = [synth.positions(n, seed) for n, seed in [(1, 3), (513, 4), (3000, 5)]]
    idx = np.concatenate([np.full(300, 5, np.uint16), np.full(257, 11339, np.uint16)])
    cases.append(synth.Positions(idx, np.array([0, 300, 557, 557, 557], np.uint32)))
    for pos in cases:
        st, ref = oracle.q_forward(w, pos)[:2]
        st2, fast = oracle.q_forward_mt(w, pos, 3)
        assert st == st2 == 0
        np.testing.assert_array_equal(fast, ref)
