"""Regenerates tests/golden/golden.npz.

The fixtures pin (a) the synthetic workload generators (SplitMix64 streams,
seeds 1 and 2) by hashes of what they produce, and (b) the oracle's outputs
on small batches of every path, so a change in either shows up as a fixture
mismatch.  The feature-pool and sparse-pool cases use the exact fixtures of
the reference's own tests (src/az/fused_feature_pool.rs:611-686: ramp tables,
hand-packed items, gradient of sum_all); the fused-policy case those of
src/az/fused_policy.rs:536-572.

Run from the repository root:  python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from chineseai_b200 import synth  # noqa: E402

PAD = 0xFFFFFFFF


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def pack_feature(feature, us, them):
    """pack_feature, src/az/fused_feature_pool.rs:130-132."""
    return feature | (us << 11) | (them << 15)


def pool_fixture():
    hidden = 7
    tables = ((np.arange(1545 * hidden, dtype=np.float32) - 4000.0) * np.float32(0.0001)).reshape(1545, hidden)
    items = np.array([pack_feature(0, 1, 8), pack_feature(95, 3, 4), PAD,
                      pack_feature(1259, 8, 0), pack_feature(95, 3, 4), pack_feature(611, 2, 6)],
                     dtype=np.uint32).reshape(2, 3)
    return tables.astype(np.float32), items


def sparse_fixture():
    rows, hidden = 11, 7
    table = ((np.arange(rows * hidden, dtype=np.float32) - 30.0) * np.float32(0.01)).reshape(rows, hidden)
    items = np.array([1, 4, PAD, 1, 10, 3, 3, PAD], dtype=np.uint32).reshape(2, 4)
    return table.astype(np.float32), items


def pack_policy_item(move_index, from_, to, captured, move_valid, capture_valid):
    """pack_policy_item, src/az/fused_policy.rs:146-157 (policy_valid set)."""
    return (move_index | from_ << 12 | to << 23 | captured << 34 | int(move_valid) << 45
            | int(capture_valid) << 46 | 1 << 47)


def policy_fixture():
    """The fused-policy test inputs of src/az/fused_policy.rs:536-572: ramp
    tables ((i % 97) - 48) * 0.001, context (i - 12) * 0.01 for two boards,
    six items (a capture, a quiet move, padding, a bias-only item, two more);
    the gradient is that of sum_all (all-ones output gradient)."""
    i = np.arange(182886)
    tables = (np.float32(1) * (i % 97).astype(np.float32) - np.float32(48.0)) * np.float32(0.001)
    c = np.arange(2 * 48)
    context = ((c.astype(np.float32) - np.float32(12.0)) * np.float32(0.01)).reshape(2, 48)
    items = np.array([pack_policy_item(3, 10, 11, 20, True, True),
                      pack_policy_item(7, 30, 40, 0, True, False),
                      0,
                      pack_policy_item(3, 0, 0, 0, False, False),
                      pack_policy_item(100, 500, 501, 0, True, False),
                      pack_policy_item(7, 30, 40, 20, True, True)], dtype=np.int64).reshape(2, 3)
    return tables.astype(np.float32), context.astype(np.float32), items


def main():
    out = {}
    qw = synth.quantized_weights(2)
    for f in qw.FIELDS:
        out[f"qw_sha_{f}"] = np.array(sha(getattr(qw, f)))
    fw = synth.float_weights(2)
    for f in fw.FIELDS:
        out[f"fw_sha_{f}"] = np.array(sha(getattr(fw, f)))

    pos = synth.positions(32, 1)
    out["q_idx"], out["q_off"] = pos.indices, pos.offsets
    st, scores, acc = oracle.q_forward(qw, pos, with_acc=True)
    assert st == 0
    out["q_scores"], out["q_acc_sha"] = scores, np.array(sha(acc))
    big = synth.positions(65536, 1)
    out["q_big_idx_sha"], out["q_big_off_sha"] = np.array(sha(big.indices)), np.array(sha(big.offsets))

    ub = synth.update_batch(32, 1)
    for f in ("parent", "flags", "rem", "rem_offsets", "add", "add_offsets", "count0"):
        out[f"u_{f}"] = getattr(ub, f)
    st, child, uscores = oracle.q_update(qw, ub)
    assert st == 0
    out["u_scores"], out["u_child_sha"] = uscores, np.array(sha(child))

    st, fout, _ = oracle.f_forward(fw, pos)
    assert st == 0
    out["f_out"] = fout

    tables, items = pool_fixture()
    st, pf = oracle.feature_pool_fwd(tables, items, 7)
    assert st == 0
    st, pg = oracle.feature_pool_bwd(items, np.ones((2, 7), np.float32), 7)
    assert st == 0
    out["pool_items"], out["pool_fwd"], out["pool_bwd"] = items, pf, pg

    table, sitems = sparse_fixture()
    st, sf = oracle.sparse_pool_fwd(table, sitems)
    assert st == 0
    st, sg = oracle.sparse_pool_bwd(sitems, np.ones((2, 7), np.float32), 11)
    assert st == 0
    out["sparse_items"], out["sparse_fwd"], out["sparse_bwd"] = sitems, sf, sg

    ptab, pctx, pitems = policy_fixture()
    st, pol = oracle.policy_fused_fwd(ptab, pctx, pitems)
    assert st == 0
    st, pgt, pgc = oracle.policy_fused_bwd(ptab, pctx, pitems, np.ones((2, 3), np.float32))
    assert st == 0
    nz = np.flatnonzero(pgt)
    out["policy_fwd"], out["policy_grad_idx"], out["policy_grad_val"] = pol, nz, pgt[nz]
    out["policy_grad_context"] = pgc

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
