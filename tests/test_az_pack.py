"""The native training batch packer (cnnue_az_pack_batch) against the
oracle's Python restatement of PackedBatch::from_indices
(src/az/dataloader.rs:113-336): every array bit for bit, with row subsets,
thread counts and the padding / filtering edge cases of the synthetic
samples."""
import numpy as np
import pytest

from chineseai_b200 import az_train
from oracle import az_pack


@pytest.fixture(scope="module")
def samples():
    return az_train.random_samples(120, 11)


@pytest.mark.parametrize("rows,threads", [(None, 1), (None, 4), ("subset", 3)])
def test_pack_matches_oracle(samples, rows, threads):
    if rows == "subset":
        rows = np.random.default_rng(3).permutation(samples.n)[:37]
    got = az_train.pack_batch(samples, rows, n_threads=threads)
    ref = az_pack.pack(samples, rows)
    for name, want in ref.items():
        have = getattr(got, name)
        assert have.shape == want.shape, name
        np.testing.assert_array_equal(have, want, err_msg=name)


def test_edge_cases_present(samples):
    b = az_train.pack_batch(samples)
    assert (b.feature_items == 0xFFFFFFFF).any()
    valid = (b.policy_items >> 47) & 1
    move_valid = (b.policy_items >> 45) & 1
    assert ((valid == 1) & (move_valid == 0)).any()  # a move with no own piece on its source
    assert ((b.policy_items >> 46) & 1).any()  # captures
    assert (b.value_wdl[:, 1] == 1.0).any()  # all-zero WDL -> draw
    assert b.values.min() >= -1.0 and b.values.max() <= 1.0
    assert np.allclose(b.policy_targets.sum(1), 1.0, atol=1e-5)
    assert (b.policy_weights >= 0).all() and (b.value_weights >= 0).all()


def test_capacity_growth_and_empty():
    s = az_train.random_samples(5, 2, max_moves=60)
    b = az_train.pack_batch(s, caps=(1, 1, 1))
    assert b.policy_items.shape[1] >= 1 and b.feature_items.shape[1] >= 1
    e = az_train.pack_batch(s, rows=np.zeros(0, np.int64))
    assert e.batch_size == 0


def test_compact_pack_shares_everything_but_the_lookups(samples):
    full = az_train.pack_batch(samples, caps=(40, 96, 96), fixed=True)
    comp = az_train.pack_batch(samples, caps=(40, 96, 96), fixed=True, compact=True)
    assert comp.compact and not full.compact
    for name in ("feature_items", "value_threat_indices", "policy_items", "policy_targets", "value_wdl", "values",
                 "rule_context", "policy_weights", "value_weights", "value_phase_masks"):
        np.testing.assert_array_equal(getattr(comp, name), getattr(full, name), err_msg=name)
    live = ((full.policy_items >> 45) & 1) == 1
    # the signature is the tactical index's low 6 bits on live moves, 0 elsewhere
    np.testing.assert_array_equal(comp.policy_signature[live], full.policy_tactical_indices[..., 1][live] & 63)
    assert (comp.policy_signature[~live] == 0).all()
    us = comp.king_buckets & 15
    them = comp.king_buckets >> 4
    assert (us <= 8).all() and (them <= 8).all()
