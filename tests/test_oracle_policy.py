"""The policy-op oracle pinned without a GPU: on the reference test's inputs
(src/az/fused_policy.rs:536-572) the C restatement equals an independent
scalar float32 restatement of the Rust loops bit for bit, and its backward
equals float64 autograd of the forward within the reference test's 3e-5;
the table op's backward equals numpy's in-order np.add.at."""
import os

import numpy as np
import pytest
import torch

import oracle
from tests.golden.make_golden import pack_policy_item, policy_fixture

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
F = np.float32


def scalar_fwd(t, c, items):
    """FusedPolicy::cpu_fwd (src/az/fused_policy.rs:178-241), one float32
    operation at a time."""
    batch, moves = items.shape
    out = np.zeros((batch, moves), np.float32)
    for b in range(batch):
        for m in range(moves):
            p = int(items[b, m]) & (2**64 - 1)
            if not (p >> 47) & 1:
                continue
            mv, fr, to, cp = p & 0xfff, (p >> 12) & 0x7ff, (p >> 23) & 0x7ff, (p >> 34) & 0x7ff
            cap = (p >> 46) & 1
            v = F(t[40352 + mv])
            if (p >> 45) & 1:
                for h in range(32):
                    d = F(t[to * 32 + h] - t[fr * 32 + h])
                    if cap:
                        d = F(d - t[cp * 32 + h])
                    v = F(v + F(d * t[40320 + h]))
                for h in range(16):
                    v = F(v + F(c[b, h] * t[42438 + mv * 16 + h]))
                for h in range(32):
                    a = F(F(c[b, 16 + h] + t[75814 + to * 32 + h]) - t[75814 + fr * 32 + h])
                    if cap:
                        a = F(a - t[75814 + cp * 32 + h])
                    v = F(v + F(a * t[116134 + mv * 32 + h]))
            out[b, m] = v
    return out


def torch_fwd(t, c, items):
    """The same forward vectorised in torch (float64) for autograd."""
    batch, moves = items.shape
    rows = []
    for b in range(batch):
        for m in range(moves):
            p = int(items[b, m]) & (2**64 - 1)
            if not (p >> 47) & 1:
                rows.append(t.new_zeros(()))
                continue
            mv, fr, to, cp = p & 0xfff, (p >> 12) & 0x7ff, (p >> 23) & 0x7ff, (p >> 34) & 0x7ff
            cap = (p >> 46) & 1
            v = t[40352 + mv]
            if (p >> 45) & 1:
                d = t[to * 32:to * 32 + 32] - t[fr * 32:fr * 32 + 32]
                if cap:
                    d = d - t[cp * 32:cp * 32 + 32]
                v = v + (d * t[40320:40352]).sum()
                v = v + (c[b, :16] * t[42438 + mv * 16:42438 + mv * 16 + 16]).sum()
                af = 75814
                a = c[b, 16:] + t[af + to * 32:af + to * 32 + 32] - t[af + fr * 32:af + fr * 32 + 32]
                if cap:
                    a = a - t[af + cp * 32:af + cp * 32 + 32]
                v = v + (a * t[116134 + mv * 32:116134 + mv * 32 + 32]).sum()
            rows.append(v)
    return torch.stack(rows).reshape(batch, moves)


def test_reference_fixture_forward_bit_exact_against_scalar_restatement():
    t, c, items = policy_fixture()
    st, out = oracle.policy_fused_fwd(t, c, items)
    assert st == 0
    np.testing.assert_array_equal(out, scalar_fwd(t, c, items))
    np.testing.assert_array_equal(out, np.load(GOLDEN)["policy_fwd"])
    assert out[0, 2] == 0.0  # padding item


def test_reference_fixture_gradient_against_autograd():
    t, c, items = policy_fixture()
    st, gt, gc = oracle.policy_fused_bwd(t, c, items, np.ones((2, 3), np.float32))
    assert st == 0
    tt = torch.tensor(t, dtype=torch.float64, requires_grad=True)
    ct = torch.tensor(c, dtype=torch.float64, requires_grad=True)
    torch_fwd(tt, ct, items).sum().backward()
    np.testing.assert_allclose(gt, tt.grad.numpy(), atol=3e-5, rtol=0)
    np.testing.assert_allclose(gc, ct.grad.numpy(), atol=3e-5, rtol=0)
    g = np.load(GOLDEN)
    full = np.zeros_like(gt)
    full[g["policy_grad_idx"]] = g["policy_grad_val"]
    np.testing.assert_array_equal(gt, full)
    np.testing.assert_array_equal(gc, g["policy_grad_context"])
    # the bias-only item (move 3, no move_valid) adds to the bias alone
    assert gt[40352 + 3] == 2.0 and gt[40352 + 7] == 2.0 and gt[40352 + 100] == 1.0


def random_policy(batch, moves, seed):
    rng = np.random.default_rng(seed)
    t = (rng.standard_normal(182886) * 0.1).astype(np.float32)
    c = rng.standard_normal((batch, 48)).astype(np.float32)
    items = np.zeros((batch, moves), np.int64)
    for b in range(batch):
        for m in range(rng.integers(0, moves + 1)):
            mv_valid = rng.random() < 0.9
            cap = mv_valid and rng.random() < 0.3
            items[b, m] = pack_policy_item(int(rng.integers(0, 2086)), int(rng.integers(0, 1260)),
                                           int(rng.integers(0, 1260)), int(rng.integers(0, 1260)), mv_valid, cap)
    return t, c, items


def test_random_gradient_against_autograd():
    t, c, items = random_policy(3, 5, 7)
    g = np.random.default_rng(8).standard_normal(items.shape).astype(np.float32)
    st, gt, gc = oracle.policy_fused_bwd(t, c, items, g)
    assert st == 0
    tt = torch.tensor(t, dtype=torch.float64, requires_grad=True)
    ct = torch.tensor(c, dtype=torch.float64, requires_grad=True)
    (torch_fwd(tt, ct, items) * torch.tensor(g, dtype=torch.float64)).sum().backward()
    np.testing.assert_allclose(gt, tt.grad.numpy(), atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(gc, ct.grad.numpy(), atol=1e-5, rtol=1e-5)
    st, out = oracle.policy_fused_fwd(t, c, items)
    np.testing.assert_array_equal(out, scalar_fwd(t, c, items))


def test_out_of_range_item_is_reported():
    t, c, items = policy_fixture()
    items = items.copy()
    items[1, 0] = pack_policy_item(2086, 1, 2, 0, True, False)  # move index past the table
    st, out = oracle.policy_fused_fwd(t, c, items)
    assert st == 2 and out[1, 0] == 0.0
    st, _, _ = oracle.policy_fused_bwd(t, c, items, np.ones((2, 3), np.float32))
    assert st == 2


@pytest.mark.parametrize("terms", [7, 2])
def test_table_op_against_numpy(terms):
    rng = np.random.default_rng(terms)
    table = rng.standard_normal(5000).astype(np.float32)
    idx = rng.integers(0, 5000, size=(4, 9, terms)).astype(np.int64)
    idx[0, 0, :] = 17  # repeated entries inside one output
    st, out = oracle.policy_table_fwd(table, idx)
    assert st == 0
    ref = np.full(idx.shape[:2], -0.0, np.float32)
    for k in range(terms):
        ref = ref + table[idx[..., k]]
    np.testing.assert_array_equal(out, ref)
    g = rng.standard_normal(idx.shape[:2]).astype(np.float32)
    st, grad = oracle.policy_table_bwd(idx, g, 5000)
    assert st == 0
    ref = np.zeros(5000, np.float32)
    np.add.at(ref, idx.reshape(-1), np.repeat(g.reshape(-1), terms))
    np.testing.assert_array_equal(grad, ref)


def test_table_op_bad_index_reported():
    table = np.ones(10, np.float32)
    idx = np.array([[[1, 12]], [[-1, 3]]], np.int64)
    st, out = oracle.policy_table_fwd(table, idx)
    assert st == 2 and out.tolist() == [[1.0], [1.0]]
