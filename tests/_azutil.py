"""Shared helpers of the AZ-NNUE tests (test infrastructure)."""
import numpy as np

from chineseai_b200 import az


def trained_like(weights: "az.AzWeights", seed: int) -> None:
    """Fills the tensors AzNnue::random leaves at zero (structural tables,
    hidden bias, rule context, value head bias and output) with seeded values,
    so every row of the trunk and every term of the value head is exercised."""
    rng = np.random.default_rng(seed)
    h = weights.hidden
    for name, scale in (("input_piece_hidden", 0.05), ("input_rank_hidden", 0.05), ("input_file_hidden", 0.05),
                        ("input_king_piece_hidden", 0.05), ("rule_context_hidden", 0.1), ("hidden_bias", 0.1),
                        ("value_head_bias", 0.1), ("value_head_output", 0.5)):
        t = weights.tensor(name)
        t[...] = rng.standard_normal(t.shape).astype(np.float32) * np.float32(scale)
    # input_hidden keeps its random-init values; scale it up a little so the
    # RMSNorm input is not dominated by the bias.
    ih = weights.tensor("input_hidden")
    ih *= np.float32(4.0)
    assert weights.hidden == h


def random_item_lists(n_lists: int, seed: int, max_len: int = 70, empty_every: int = 9):
    """Ragged lists of valid packed items (not from a board): lengths 0..max_len,
    every `empty_every`-th list empty, features < 1260, buckets 0..8."""
    rng = np.random.default_rng(seed)
    lists = []
    for i in range(n_lists):
        n = 0 if i % empty_every == 0 else int(rng.integers(1, max_len + 1))
        f = rng.integers(0, 1260, n, dtype=np.uint32)
        us = rng.integers(0, 9, n, dtype=np.uint32)
        them = rng.integers(0, 9, n, dtype=np.uint32)
        lists.append((f | (us << 11) | (them << 15)).astype(np.uint32))
    return lists


def trained_policy(weights: "az.AzWeights", seed: int) -> None:
    """Seeded values for the policy tensors the quantiser reads (move table,
    sparse table and factors) and a re-quantisation."""
    rng = np.random.default_rng(seed)
    for name, scale in (("policy_accumulator_move", 1.0), ("policy_sparse_table", 0.1),
                        ("policy_sparse_factor", 0.1)):
        t = weights.tensor(name)
        t[...] = rng.standard_normal(t.shape).astype(np.float32) * np.float32(scale)
    weights.quantize()


def full_policy(weights: "az.AzWeights", seed: int) -> None:
    """Seeded values for every policy-head and threat tensor, so each term of
    the policy logit and both optional branches (threat, tactical) are live."""
    rng = np.random.default_rng(seed)
    for name, scale in (("policy_move_bias", 0.3), ("policy_consequence_output", 0.3),
                        ("policy_move_context", 0.3), ("policy_accumulator_move", 1.0),
                        ("policy_sparse_table", 0.1), ("policy_sparse_factor", 0.1), ("policy_tactical", 0.2),
                        ("value_threat_output", 0.5), ("policy_threat_context", 0.2)):
        t = weights.tensor(name)
        t[...] = rng.standard_normal(t.shape).astype(np.float32) * np.float32(scale)
    weights.quantize()
