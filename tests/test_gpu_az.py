"""GPU parity of the reference-native AZ-NNUE evaluator against the oracle.

Refresh and transition are bit-identical to the oracle (the reference's row
order, one fp32 add per row per column); the value head is within 1e-4 of it
(the reference's dot products run in another summation order).  Cases: board
lists of random positions, ragged synthetic lists (empty, > 32 items), hidden
sizes on both the float4 and the scalar column paths, bad items and offsets,
in-place transitions, the reference's incremental-equals-refresh walk
(src/az.rs:3470-3495) and its neutral-initial-value check
(src/az.rs:3354-3363)."""
import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import az
from chineseai_b200.quantized import as_device

from ._azutil import random_item_lists, trained_like

pytestmark = pytest.mark.gpu

_MODELS = {}


def _model(hidden, seed=20260807):
    key = (hidden, seed)
    if key not in _MODELS:
        w = az.AzWeights.random(hidden, seed)
        trained_like(w, seed % 1000)
        _MODELS[key] = (w, w.tensors(), az.AzModel(w, device=0))
    return _MODELS[key]


def _dev(a):
    return as_device(np.ascontiguousarray(a), torch.device("cuda", 0))


@pytest.mark.parametrize("hidden", [128, 256, 512, 32, 16, 100, 4, 7])
def test_refresh_bit_exact_on_boards(hidden):
    w, tensors, model = _model(hidden)
    boards = az.random_boards(700, seed=hidden)
    items, offsets = az.node_lists(boards)
    acc = model.refresh(_dev(items), _dev(offsets))
    assert model.read_status() == 0
    st, ref = oracle.az_refresh(tensors, hidden, items, offsets)
    assert st == 0
    np.testing.assert_array_equal(acc.cpu().numpy(), ref)


@pytest.mark.parametrize("hidden", [128, 20])
def test_refresh_bit_exact_on_ragged_lists(hidden):
    w, tensors, model = _model(hidden)
    lists = random_item_lists(1500, seed=5, max_len=90)
    items, offsets = az.pack_lists(lists)
    acc = model.refresh(_dev(items), _dev(offsets))
    assert model.read_status() == 0
    st, ref = oracle.az_refresh(tensors, hidden, items, offsets)
    np.testing.assert_array_equal(acc.cpu().numpy(), ref)
    # an empty list is the hidden bias
    np.testing.assert_array_equal(acc[0].cpu().numpy(), w.tensor("hidden_bias"))


def test_refresh_flags_bad_items_and_skips_them():
    w, tensors, model = _model(128)
    lists = random_item_lists(64, seed=6, max_len=40, empty_every=1000)
    lists[3][2] = 1300                      # feature >= 1260
    lists[10][0] = 5 | (9 << 11)            # us bucket 9
    lists[20][5] = 7 | (3 << 11) | (12 << 15)  # them bucket 12
    items, offsets = az.pack_lists(lists)
    acc = model.refresh(_dev(items), _dev(offsets))
    assert model.read_status() == 2  # CNNUE_ERR_BAD_INDEX
    st, ref = oracle.az_refresh(tensors, 128, items, offsets)
    assert st == 2
    np.testing.assert_array_equal(acc.cpu().numpy(), ref)
    bad = offsets.copy()
    bad[5] = bad[6] + 1  # not monotone
    model.refresh(_dev(items), _dev(bad))
    assert model.read_status() == 3  # CNNUE_ERR_BAD_OFFSETS
    assert model.read_status() == 0  # read clears


def _moves(boards, seed):
    rng = np.random.default_rng(seed)
    deltas, refresh, lists, afters = [], [], [], []
    for b in boards:
        frm, to = az.random_move(b, rng)
        afters.append(az.apply_move(b, frm, to))
        for p in (0, 1):
            m = az.move_items(b, frm, to, p)
            deltas.append(m.delta)
            refresh.append(m.refresh)
            lists.append(m.items)
    items, offsets = az.pack_lists(lists)
    return np.stack(deltas), np.array(refresh, np.uint8), items, offsets, np.stack(afters)


@pytest.mark.parametrize("hidden", [128, 512, 16, 7])
def test_transition_bit_exact(hidden):
    w, tensors, model = _model(hidden)
    boards = az.random_boards(800, seed=100 + hidden)
    p_items, p_off = az.node_lists(boards)
    parent = model.refresh(_dev(p_items), _dev(p_off))
    delta, refresh, items, offsets, afters = _moves(boards, seed=hidden)
    assert 0 < refresh.sum() < len(refresh)
    child = model.transition(parent, _dev(delta), _dev(refresh), _dev(items), _dev(offsets))
    assert model.read_status() == 0
    st, ref = oracle.az_transition(tensors, hidden, parent.cpu().numpy(), delta, refresh, items, offsets)
    assert st == 0
    np.testing.assert_array_equal(child.cpu().numpy(), ref)
    # in place gives the same bits
    model.transition(parent, _dev(delta), _dev(refresh), _dev(items), _dev(offsets), out=parent)
    np.testing.assert_array_equal(parent.cpu().numpy(), ref)
    # and the incremental child is the refresh of the child board within 2e-5
    full = model.refresh(*[_dev(a) for a in az.node_lists(afters)])
    assert (parent - full).abs().max().item() < 2e-5


def test_transition_without_refresh_lists_takes_null_items():
    w, tensors, model = _model(128)
    boards = az.random_boards(300, seed=77)
    parent = model.refresh(*[_dev(a) for a in az.node_lists(boards)])
    delta, refresh, items, offsets, _ = _moves(boards, seed=78)
    keep = refresh == 0
    delta, parent_k = delta[keep], parent[torch.from_numpy(keep).cuda()]
    zeros = np.zeros(len(delta), np.uint8)
    child = model.transition(parent_k, _dev(delta), _dev(zeros))
    assert model.read_status() == 0
    st, ref = oracle.az_transition(tensors, 128, parent_k.cpu().numpy(), delta, zeros, np.zeros(0, np.uint32),
                                   np.zeros(len(delta) + 1, np.uint32))
    np.testing.assert_array_equal(child.cpu().numpy(), ref)
    # a refresh flag with no item lists is reported, not read
    zeros[0] = 1
    model.transition(parent_k, _dev(delta), _dev(zeros))
    assert model.read_status() == 3


def test_incremental_walk_matches_refresh():
    """src/az.rs:3470-3495 on the device: 32 moves from the start position."""
    w, tensors, model = _model(128)
    rng = np.random.default_rng(21)
    board, _ = az.board_from_fen(az.STARTPOS)
    acc = model.refresh(*[_dev(a) for a in az.node_lists(board[None])])
    for ply in range(32):
        frm, to = az.random_move(board, rng, side=ply % 2)
        ms = [az.move_items(board, frm, to, p) for p in (0, 1)]
        r_items, r_off = az.pack_lists([m.items for m in ms])
        acc = model.transition(acc, _dev(np.stack([m.delta for m in ms])),
                               _dev(np.array([m.refresh for m in ms], np.uint8)), _dev(r_items), _dev(r_off))
        board = az.apply_move(board, frm, to)
        full = model.refresh(*[_dev(a) for a in az.node_lists(board[None])])
        assert (acc - full).abs().max().item() < 2e-5
    assert model.read_status() == 0


@pytest.mark.parametrize("hidden", [128, 512, 32, 7])
def test_value_matches_oracle(hidden):
    w, tensors, model = _model(hidden)
    boards = az.random_boards(1001, seed=200 + hidden)
    acc = model.refresh(*[_dev(a) for a in az.node_lists(boards)])
    rng = np.random.default_rng(hidden)
    side = rng.integers(0, 2, len(boards)).astype(np.uint8)
    rule = (rng.random((len(boards), 7)) * (rng.random((len(boards), 7)) < 0.4)).astype(np.float32)
    threat = rng.standard_normal((len(boards), 3)).astype(np.float32)
    wdl, q = model.value(acc, side=_dev(side), rule=_dev(rule), threat=_dev(threat))
    a = acc.cpu().numpy().reshape(len(boards), 2, hidden)
    stm = a[np.arange(len(boards)), side]
    ref_wdl, ref_q = oracle.az_value(tensors, hidden, stm, rule, threat)
    np.testing.assert_allclose(wdl.cpu().numpy(), ref_wdl, atol=1e-4, rtol=0)
    np.testing.assert_allclose(q.cpu().numpy(), ref_q, atol=1e-4, rtol=0)
    assert np.abs(ref_q).max() > 0.05  # the head is not trivially neutral here
    # [n][H] layout without rule or threat
    wdl2, q2 = model.value(torch.from_numpy(stm).cuda())
    r2_wdl, r2_q = oracle.az_value(tensors, hidden, stm)
    np.testing.assert_allclose(q2.cpu().numpy(), r2_q, atol=1e-4, rtol=0)
    np.testing.assert_allclose(wdl2.sum(1).cpu().numpy(), 1.0, atol=1e-5)


def test_random_init_value_is_neutral():
    """src/az.rs:3354-3363: AzNnue::random(512, 20260409) evaluates startpos to 0."""
    w = az.AzWeights.random(512, 20260409)
    model = az.AzModel(w, device=0)
    try:
        board, side = az.board_from_fen(az.STARTPOS)
        acc = model.refresh(*[_dev(a) for a in az.node_lists(board[None])])
        wdl, q = model.value(acc, side=_dev(np.array([side], np.uint8)))
        assert abs(q.item()) < 1e-6
        np.testing.assert_allclose(wdl.cpu().numpy(), 1.0 / 3.0, atol=1e-6)
    finally:
        model.close()


# ---- int16 policy accumulator (bit-exact) -----------------------------------
_POLICY = {}


def _policy_model():
    if "m" not in _POLICY:
        from ._azutil import trained_policy
        w = az.AzWeights.random(128, 20260817)
        trained_like(w, 31)
        trained_policy(w, 32)
        fq, _ = w.quant_table(az.Q_POLICY_FEATURE)
        _POLICY["m"] = (w, fq, az.AzModel(w, device=0))
    return _POLICY["m"]


def test_policy_refresh_bit_exact():
    w, fq, model = _policy_model()
    boards = az.random_boards(1500, seed=41)
    items, offsets = az.node_lists(boards)
    acc = model.policy_refresh(_dev(items), _dev(offsets))
    assert model.read_status() == 0
    st, ref = oracle.az_policy_refresh(fq, items, offsets)
    assert st == 0
    np.testing.assert_array_equal(acc.cpu().numpy(), ref)


def _hottest_item(fq):
    """The packed item whose 6 policy rows have the largest |sum| at one rank."""
    q = fq.astype(np.int32)
    f = np.arange(1260)
    piece, sq = f // 90, f % 90
    base = q[f] + q[1260 + piece] + q[1274 + sq // 9] + q[1284 + sq % 9]  # [1260][32]
    best, best_item = -1, 0
    for us in range(9):
        for them in range(9):
            tot = base + q[1293 + us * 14 + piece] + q[1293 + (9 + them) * 14 + piece]
            i = int(np.argmax(np.abs(tot).max(axis=1)))
            v = int(np.abs(tot[i]).max())
            if v > best:
                best, best_item = v, i | (us << 11) | (them << 15)
    assert best * 90 > 32767
    return np.uint32(best_item)


def test_policy_refresh_saturates_like_the_reference():
    """Lists of 90 copies of the item whose rows hold +-127 push int16 past its
    range; each row add clamps, in order, as add_quantized_policy_row does."""
    w, fq, model = _policy_model()
    hot = _hottest_item(fq)
    lists = random_item_lists(300, seed=42, max_len=90)
    for i in range(0, 300, 3):
        lists[i] = np.full(90, hot, np.uint32)
    items, offsets = az.pack_lists(lists)
    acc = model.policy_refresh(_dev(items), _dev(offsets))
    st, ref = oracle.az_policy_refresh(fq, items, offsets)
    assert model.read_status() == 0 and st == 0
    assert (np.abs(ref.astype(np.int32)) == 32767).any() or (ref == -32768).any()
    np.testing.assert_array_equal(acc.cpu().numpy(), ref)
    # transitions from saturated parents
    delta = np.tile(np.array([hot, az.NO_ITEM, hot], np.uint32), (len(lists), 1))
    delta[1::2, 1] = hot
    refresh = np.zeros(len(lists), np.uint8)
    child = model.policy_transition(acc, _dev(delta), _dev(refresh))
    st, ref2 = oracle.az_policy_transition(fq, ref, delta, refresh, np.zeros(0, np.uint32),
                                           np.zeros(len(lists) + 1, np.uint32))
    np.testing.assert_array_equal(child.cpu().numpy(), ref2)


def test_policy_transition_bit_exact_and_in_place():
    w, fq, model = _policy_model()
    boards = az.random_boards(1200, seed=43)
    parent = model.policy_refresh(*[_dev(a) for a in az.node_lists(boards)])
    delta, refresh, items, offsets, afters = _moves(boards, seed=44)
    child = model.policy_transition(parent, _dev(delta), _dev(refresh), _dev(items), _dev(offsets))
    assert model.read_status() == 0
    st, ref = oracle.az_policy_transition(fq, parent.cpu().numpy(), delta, refresh, items, offsets)
    np.testing.assert_array_equal(child.cpu().numpy(), ref)
    model.policy_transition(parent, _dev(delta), _dev(refresh), _dev(items), _dev(offsets), out=parent)
    np.testing.assert_array_equal(parent.cpu().numpy(), ref)
    # equals the refresh of the child boards exactly (no saturation at <= 32 pieces)
    full = model.policy_refresh(*[_dev(a) for a in az.node_lists(afters)])
    assert torch.equal(parent, full)


def test_policy_walk_matches_refresh_exactly():
    """src/az.rs:3497-3527 on the device."""
    w, fq, model = _policy_model()
    rng = np.random.default_rng(45)
    board, _ = az.board_from_fen(az.STARTPOS)
    acc = model.policy_refresh(*[_dev(a) for a in az.node_lists(board[None])])
    for ply in range(32):
        frm, to = az.random_move(board, rng, side=ply % 2)
        ms = [az.move_items(board, frm, to, p) for p in (0, 1)]
        r_items, r_off = az.pack_lists([m.items for m in ms])
        acc = model.policy_transition(acc, _dev(np.stack([m.delta for m in ms])),
                                      _dev(np.array([m.refresh for m in ms], np.uint8)), _dev(r_items), _dev(r_off))
        board = az.apply_move(board, frm, to)
        full = model.policy_refresh(*[_dev(a) for a in az.node_lists(board[None])])
        assert torch.equal(acc, full)
    assert model.read_status() == 0


# ---- threat logits (bit-exact) ---------------------------------------------
def test_threat_logits_bit_exact_and_value_with_threat():
    w = az.AzWeights.random(128, 20260807)
    trained_like(w, 51)
    rng = np.random.default_rng(52)
    out = w.tensor("value_threat_output")
    out[...] = rng.standard_normal(out.shape).astype(np.float32) * np.float32(0.5)
    emb = w.tensor("value_threat_embedding")
    emb *= np.float32(20.0)  # larger rows: activations reach the clamp and the int16 sums wrap sometimes
    w.quantize()
    assert w.quant_flags()[0]
    table, scale = w.quant_table(az.Q_VALUE_THREAT)
    model = az.AzModel(w, device=0)
    try:
        boards = az.random_boards(1500, seed=53)
        side = rng.integers(0, 2, len(boards)).astype(np.uint8)
        lists = [az.threat_features(b, int(s)) for b, s in zip(boards, side)]
        lists[7] = np.zeros(0, np.uint32)  # no attacks
        lists[9] = np.tile(lists[9], 40) if len(lists[9]) else np.full(200, 5, np.uint32)  # long: wraps
        feats, offs = az.pack_lists(lists)
        logits = model.threat_logits(_dev(feats), _dev(offs))
        assert model.read_status() == 0
        st, ref = oracle.az_threat_logits(table, scale, w.tensor("value_threat_output"), feats, offs)
        assert st == 0
        np.testing.assert_array_equal(logits.cpu().numpy(), ref)
        # the value head with these threat logits agrees with the oracle's
        acc = model.refresh(*[_dev(a) for a in az.node_lists(boards)])
        wdl, q = model.value(acc, side=_dev(side), threat=logits)
        a = acc.cpu().numpy().reshape(len(boards), 2, 128)[np.arange(len(boards)), side]
        r_wdl, r_q = oracle.az_value(w.tensors(), 128, a, None, ref)
        np.testing.assert_allclose(q.cpu().numpy(), r_q, atol=1e-4, rtol=0)
    finally:
        model.close()


# ---- the full evaluator entry point (value + threat + policy logits) --------
def test_evaluate_matches_oracle_with_every_branch_live():
    from ._azutil import full_policy
    w = az.AzWeights.random(128, 20260819)
    trained_like(w, 61)
    full_policy(w, 62)
    assert w.quant_flags() == (True, True)
    t = w.tensors()
    quant = oracle.az_quantize(t, 128)
    model = az.AzModel(w, device=0)
    try:
        rng = np.random.default_rng(63)
        boards = az.random_boards(600, seed=64)
        side = rng.integers(0, 2, len(boards)).astype(np.uint8)
        acc = model.refresh(*[_dev(a) for a in az.node_lists(boards)])
        pacc = model.policy_refresh(*[_dev(a) for a in az.node_lists(boards)])
        tf, to = az.pack_lists([az.threat_features(b, int(s)) for b, s in zip(boards, side)])
        move_lists = [az.pseudo_moves(b, int(s), rng, 40) for b, s in zip(boards, side)]
        infos = [az.policy_moves(b, int(s), m) for b, s, m in zip(boards, side, move_lists)]
        offs = np.zeros(len(boards) + 1, np.uint32)
        offs[1:] = np.cumsum([len(i) for i in infos])
        info = np.concatenate(infos).astype(np.uint32)
        rule = (rng.random((len(boards), 7)) * (rng.random((len(boards), 7)) < 0.3)).astype(np.float32)
        wdl, q, logits = model.evaluate(acc, side=_dev(side), rule=_dev(rule), threat_features=_dev(tf),
                                        threat_offsets=_dev(to), policy_acc=pacc, move_info=_dev(info),
                                        move_offsets=_dev(offs))
        assert model.read_status() == 0
        # oracle: threat logits + activations, value with the normalised hidden, policy logits
        a = acc.cpu().numpy().reshape(len(boards), 2, 128)[np.arange(len(boards)), side]
        pa = pacc.cpu().numpy().reshape(len(boards), 2, 32)[np.arange(len(boards)), side]
        st, tl, act = oracle.az_threat_logits(quant["value_threat"], float(quant["scales"][3]), t[11], tf, to,
                                              with_act=True)
        r_wdl, r_q, x = oracle.az_value(t, 128, a, rule, tl, with_x=True)
        r_logits = oracle.az_policy_logits(t, 128, quant, True, x, act, pa, info, offs)
        np.testing.assert_allclose(q.cpu().numpy(), r_q, atol=1e-4, rtol=0)
        np.testing.assert_allclose(wdl.cpu().numpy(), r_wdl, atol=1e-4, rtol=0)
        g = logits.cpu().numpy()
        assert np.abs(r_logits).max() > 1.0
        np.testing.assert_allclose(g, r_logits, atol=1e-4, rtol=1e-5)
    finally:
        model.close()
