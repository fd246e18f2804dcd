"""CPU tests of the AZ-NNUE host side: FEN parsing and feature items against
the reference's own known answers (src/nnue.rs:91-129), AzNnue::random against
the oracle and an independent SplitMix64, the safetensors weight file against
the `safetensors` package (the library the reference's Candle uses to write
it), and the move deltas of apply_transition_for_perspective."""
import os

import numpy as np
import pytest

import oracle
from chineseai_b200 import az
from chineseai_b200._lib import CnnueError

from ._azutil import trained_like


def test_known_answer_side_to_move_canonical_features():
    # src/nnue.rs:91-119: Black to move; our general on square 4, theirs on 85.
    board, side = az.board_from_fen("4k4/9/9/9/4p4/9/9/9/9/4K4 b - - 0 1")
    assert side == 1
    feats = az.features(board, side) & 0x7FF
    us_general = 0 * 90 + (89 - 4)
    them_general = 7 * 90 + (89 - 85)
    assert us_general == 85 and them_general == 634
    assert us_general in feats and them_general in feats
    assert len(feats) == 3


def test_known_answer_startpos_has_32_features():
    # src/nnue.rs:121-129
    board, side = az.board_from_fen(az.STARTPOS)
    assert side == 0
    feats = az.features(board, 0) & 0x7FF
    assert len(feats) == 32 and feats.max() < 1260
    # both generals on their home squares -> bucket (9-7)*3 + (4-3) = 7
    items = az.features(board, 0)
    assert set((items >> 11) & 0xF) == {7} and set((items >> 15) & 0xF) == {7}


@pytest.mark.parametrize("fen", ["rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKAXNR w",
                                 "rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9 w",
                                 "rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR x",
                                 "rnbakabnrr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR w",
                                 "rnbakabn/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR w"])
def test_malformed_fen_is_a_format_error(fen):
    with pytest.raises(CnnueError) as e:
        az.board_from_fen(fen)
    assert e.value.status == 6


def test_fen_alias_letters_and_default_side():
    a, sa = az.board_from_fen("rheakaehr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RHEAKAEHR")
    b, sb = az.board_from_fen(az.STARTPOS)
    assert sa == 0 and np.array_equal(a, b)


def test_features_match_oracle_on_random_boards():
    boards = az.random_boards(300, seed=11)
    boards[:20] = az.random_boards(20, seed=12, generals=False)  # generals absent -> bucket 4
    for b in boards:
        for p in (0, 1):
            np.testing.assert_array_equal(az.features(b, p), oracle.az_features(b, p))


def _splitmix_weights(seed: int, n: int, scale: float) -> np.ndarray:
    """Independent restatement of SplitMix64::weight (src/az.rs:3146-3176)."""
    m = (1 << 64) - 1
    state, out = seed, []
    for _ in range(n):
        v = (state + 0x9E3779B97F4A7C15) & m
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m
        state = v ^ (v >> 31)
        u = np.float32((state >> 11) * (1.0 / (1 << 53)))
        out.append((u * np.float32(2.0) - np.float32(1.0)) * np.float32(scale))
    return np.array(out, np.float32)


@pytest.mark.parametrize("hidden,seed", [(4, 7), (16, 12345), (128, 20260807)])
def test_random_weights_match_oracle_and_splitmix(hidden, seed):
    w = az.AzWeights.random(hidden, seed)
    ref = oracle.az_random(hidden, seed)
    for i in range(az.N_TENSORS):
        np.testing.assert_array_equal(w.tensor(i).reshape(-1), ref[i], err_msg=w.names[i])
    np.testing.assert_array_equal(w.tensor(0).reshape(-1)[:64], _splitmix_weights(seed, 64, 0.015))
    # every tensor the reference leaves at zero is zero
    for i in (1, 2, 3, 4, 5, 6, 8, 9, 11, 12, 13, 14, 16, 18, 19, 20, 21):
        assert not w.tensor(i).any(), w.names[i]


def test_tensor_names_and_shapes_follow_the_reference_layout():
    w = az.AzWeights.random(32, 1)
    assert w.names[:7] == ["input_hidden", "input_piece_hidden", "input_rank_hidden", "input_file_hidden",
                           "input_king_piece_hidden", "rule_context_hidden", "hidden_bias"]
    assert w.names[-3:] == ["policy_sparse_table", "policy_sparse_factor", "policy_tactical"]
    assert w.tensor("input_king_piece_hidden").shape == (252, 32)
    assert w.tensor("value_threat_embedding").shape == (57702, 64)
    assert w.tensor("policy_sparse_table").shape == (2396815,)


def test_weight_file_round_trip_through_safetensors_package(tmp_path):
    st = pytest.importorskip("safetensors.numpy")
    w = az.AzWeights.random(16, 42)
    trained_like(w, 5)
    path = str(tmp_path / "model.safetensors")
    w.save(path)
    loaded = st.load_file(path)
    assert loaded["az_model_format_version"].tolist() == [20.0]
    for i, name in enumerate(w.names):
        assert loaded[name].dtype == np.float32 and loaded[name].shape == w.tensor(i).shape
        np.testing.assert_array_equal(loaded[name], w.tensor(i))
    # a file written by the safetensors package reads back identically
    other = str(tmp_path / "other.safetensors")
    st.save_file({k: np.ascontiguousarray(v) for k, v in loaded.items()}, other, metadata={"format": "pt"})
    w2 = az.AzWeights.load(other)
    assert w2.hidden == 16
    for i in range(az.N_TENSORS):
        np.testing.assert_array_equal(w2.tensor(i), w.tensor(i))


def _write(path, tensors):
    from safetensors.numpy import save_file
    save_file({k: np.ascontiguousarray(v) for k, v in tensors.items()}, path)


def test_weight_file_errors(tmp_path):
    pytest.importorskip("safetensors.numpy")
    from safetensors.numpy import load_file
    w = az.AzWeights.random(8, 3)
    good = str(tmp_path / "good.safetensors")
    w.save(good)
    base = load_file(good)

    def expect(tensors, status, text):
        p = str(tmp_path / "bad.safetensors")
        _write(p, tensors)
        with pytest.raises(CnnueError) as e:
            az.AzWeights.load(p)
        assert e.value.status == status and text in str(e.value), str(e.value)

    expect({**base, "az_model_format_version": np.array([19.0], np.float32)}, 6, "unsupported AZ model format")
    expect({k: v for k, v in base.items() if k != "az_model_format_version"}, 6, "az_model_format_version")
    expect({k: v for k, v in base.items() if k != "policy_tactical"}, 6, "policy_tactical")
    expect({**base, "value_head_bias": np.zeros(95, np.float32)}, 6, "value_head_bias")
    expect({**base, "input_hidden": np.zeros((1260, 9), np.float32)}, 6, "input_hidden")
    expect({**base, "hidden_bias": base["hidden_bias"].astype(np.float64)}, 6, "expected F32")
    with pytest.raises(CnnueError) as e:
        az.AzWeights.load(str(tmp_path / "missing.safetensors"))
    assert e.value.status == 7
    trunc = str(tmp_path / "trunc.safetensors")
    with open(good, "rb") as f:
        data = f.read()
    with open(trunc, "wb") as f:
        f.write(data[: len(data) // 2])
    with pytest.raises(CnnueError) as e:
        az.AzWeights.load(trunc)
    assert e.value.status == 6


def test_move_items_match_features_of_both_boards():
    rng = np.random.default_rng(3)
    boards = az.random_boards(200, seed=4)
    n_refresh = n_capture = 0
    for b in boards:
        frm, to = az.random_move(b, rng)
        after = az.apply_move(b, frm, to)
        for p in (0, 1):
            m = az.move_items(b, frm, to, p)
            before_items, after_items = az.features(b, p), az.features(after, p)
            buckets_before = ((before_items >> 11) & 0xFF)[0]
            buckets_after = ((after_items >> 11) & 0xFF)[0]
            if m.refresh:
                n_refresh += 1
                assert buckets_before != buckets_after
                np.testing.assert_array_equal(m.items, after_items)
            else:
                assert buckets_before == buckets_after
                assert m.delta[0] in before_items and m.delta[2] in after_items
                assert m.delta[0] not in after_items or b[frm] == after[frm]
                if b[to] != 0:
                    n_capture += 1
                    assert m.delta[1] in before_items
                else:
                    assert m.delta[1] == az.NO_ITEM
    assert n_refresh > 0 and n_capture > 0


def test_incremental_equals_refresh_on_the_oracle():
    """src/az.rs:3470-3495 on the oracle: 32 moves, |incremental - refresh| < 2e-5."""
    w = az.AzWeights.random(128, 20260807)
    trained_like(w, 9)
    tensors = w.tensors()
    rng = np.random.default_rng(8)
    board, _ = az.board_from_fen(az.STARTPOS)
    items, offsets = az.node_lists(board[None])
    st, acc = oracle.az_refresh(tensors, 128, items, offsets)
    assert st == 0
    for ply in range(32):
        frm, to = az.random_move(board, rng, side=ply % 2)
        ms = [az.move_items(board, frm, to, p) for p in (0, 1)]
        delta = np.stack([m.delta for m in ms])
        refresh = np.array([m.refresh for m in ms], np.uint8)
        r_items, r_off = az.pack_lists([m.items for m in ms])
        st, acc = oracle.az_transition(tensors, 128, acc, delta, refresh, r_items, r_off)
        assert st == 0
        board = az.apply_move(board, frm, to)
        st, full = oracle.az_refresh(tensors, 128, *az.node_lists(board[None]))
        assert np.abs(acc - full).max() < 2e-5


def test_random_init_value_is_neutral_on_the_oracle():
    """src/az.rs:3354-3363: zero value_head_output gives q = 0 exactly."""
    w = az.AzWeights.random(512, 20260409)
    tensors = w.tensors()
    board, side = az.board_from_fen(az.STARTPOS)
    st, acc = oracle.az_refresh(tensors, 512, *az.node_lists(board[None]))
    wdl, q = oracle.az_value(tensors, 512, acc[side][None])
    assert abs(q[0]) < 1e-6 and np.allclose(wdl, 1.0 / 3.0)


def test_device_model_rejects_bad_hidden_sizes_without_a_gpu():
    from chineseai_b200._lib import lib
    import ctypes as C
    h = C.c_void_p()
    w = az.AzWeights.random(130, 1)  # >= 128 and not a multiple of 4
    assert lib().cnnue_az_model_create(w.handle, 0, C.byref(h)) == 1
    w = az.AzWeights.random(516, 1)
    assert lib().cnnue_az_model_create(w.handle, 0, C.byref(h)) == 1


def test_dense_move_space_matches_enumeration():
    """src/az.rs:3344-3352: 2086 dense moves, dense <-> sparse inverse."""
    d2s, s2d = az.dense_moves()
    assert len(d2s) == 2086
    np.testing.assert_array_equal(d2s, oracle.az_dense_moves())
    assert all(s2d[d2s[i]] == i for i in range(2086))
    assert (s2d != 0xFFFF).sum() == 2086
    # rook lines from a corner: 8 + 9 targets; a horse step and a palace diagonal exist
    assert sum(1 for s in d2s if s // 90 == 0) == 17 + 2  # + the horse steps to (1,2) and (2,1)
    assert s2d[76 * 90 + 84] != 0xFFFF and s2d[84 * 90 + 76] != 0xFFFF  # palace diagonal (9,3) <-> (8,4)
    assert s2d[84 * 90 + 74] == 0xFFFF  # (9,3) -> (8,2) is no palace diagonal


@pytest.mark.parametrize("hidden,seed", [(128, 20260817), (16, 7), (100, 3)])
def test_quantised_tables_match_oracle(hidden, seed):
    from ._azutil import trained_policy
    w = az.AzWeights.random(hidden, seed)
    trained_like(w, seed % 97)
    trained_policy(w, seed % 89)
    ref = oracle.az_quantize(w.tensors(), hidden)
    for which, name in enumerate(["policy_feature", "policy_move", "policy_sparse", "value_threat",
                                  "moved_delta", "capture"]):
        got, scale = w.quant_table(which)
        np.testing.assert_array_equal(got.reshape(-1), ref[name].reshape(-1), err_msg=name)
        if which < 4:
            assert scale == ref["scales"][which], name
    assert list(w.quant_flags()) == [bool(x) for x in ref["flags"]]


def test_quantised_policy_rows_follow_float64_projection():
    """Independent pin of the projection: q = round(x / scale) of the float64
    dot products, except within 1e-3 of a rounding boundary."""
    w = az.AzWeights.random(128, 20260817)
    trained_like(w, 4)
    w.quantize()
    t = w.tensors()
    rows = np.concatenate([t[i].astype(np.float64) for i in (0, 1, 2, 3, 4)] + [t[6][None].astype(np.float64)])
    proj = rows @ t[17].astype(np.float64).T  # [1546][32]
    q, scale = w.quant_table(az.Q_POLICY_FEATURE)
    assert abs(scale - np.abs(proj).max() / 127) < 1e-6 * scale * 127
    x = proj / scale
    frac = np.abs(x - np.floor(x) - 0.5)
    safe = frac > 1e-3
    expect = np.clip(np.sign(x) * np.floor(np.abs(x) + 0.5), -127, 127)
    np.testing.assert_array_equal(q[safe], expect[safe])
    assert safe.mean() > 0.99


def test_random_init_quantisation_flags_and_zero_rows():
    w = az.AzWeights.random(128, 20260817)
    assert w.quant_flags() == (False, False)  # zero threat and tactical outputs
    q, _ = w.quant_table(az.Q_POLICY_FEATURE)
    assert not q[1260:].any()  # structural and bias rows are zero at init
    assert q[:1260].any()


def test_policy_accumulator_incremental_equals_refresh_on_the_oracle():
    """src/az.rs:3497-3527 on the oracle: exact equality over 32 moves."""
    from ._azutil import trained_policy
    w = az.AzWeights.random(128, 20260817)
    trained_like(w, 2)
    trained_policy(w, 3)
    fq, _ = w.quant_table(az.Q_POLICY_FEATURE)
    rng = np.random.default_rng(5)
    board, _ = az.board_from_fen(az.STARTPOS)
    st, acc = oracle.az_policy_refresh(fq, *az.node_lists(board[None]))
    assert st == 0
    for ply in range(32):
        frm, to = az.random_move(board, rng, side=ply % 2)
        ms = [az.move_items(board, frm, to, p) for p in (0, 1)]
        r_items, r_off = az.pack_lists([m.items for m in ms])
        st, acc = oracle.az_policy_transition(fq, acc, np.stack([m.delta for m in ms]),
                                              np.array([m.refresh for m in ms], np.uint8), r_items, r_off)
        board = az.apply_move(board, frm, to)
        st2, full = oracle.az_policy_refresh(fq, *az.node_lists(board[None]))
        np.testing.assert_array_equal(acc, full)


def test_threat_vocabulary_is_the_reference_size():
    """threat_relation_map enumerates exactly VALUE_THREAT_VOCAB = 57,702
    slots (src/az.rs:106, asserted at :656) - in the library and the oracle."""
    from chineseai_b200._lib import lib
    assert lib().cnnue_az_threat_vocab() == 57702
    assert oracle.az_threat_vocab() == 57702


def test_threat_features_of_the_start_position():
    """Start position, Red to move: 4 cannon-over-screen attacks on the
    opposing horses, 8 rook contacts (own horse and pawn), 4 general contacts
    (own advisors) - 16 relations."""
    board, side = az.board_from_fen(az.STARTPOS)
    f = az.threat_features(board, side)
    assert len(f) == 16 and len(set(f.tolist())) == 16
    np.testing.assert_array_equal(f, oracle.az_threat_features(board, side))
    # colour symmetry: the mirrored position seen by Black gives the same rows
    mirrored = -board[::-1].copy()
    np.testing.assert_array_equal(np.sort(az.threat_features(mirrored, 1)), np.sort(f))


def test_threat_features_match_oracle_on_random_boards():
    boards = az.random_boards(300, seed=17)
    for b in boards:
        for side in (0, 1):
            got = az.threat_features(b, side)
            np.testing.assert_array_equal(got, oracle.az_threat_features(b, side))
            assert (got < 57702).all()


def _check_bit(fen, frm, to):
    board, side = az.board_from_fen(fen)
    mv = np.array([[frm, to]], np.uint8)
    info = az.policy_moves(board, side, mv)
    np.testing.assert_array_equal(info, oracle.az_policy_moves(board, side, mv))
    return (int(info[0, 0]) >> 25) & 1


def test_gives_check_known_answers():
    """gives_check_after_move_fast (src/xiangqi/mod.rs:763-831) on hand-made
    positions: a rook onto the general's open file, a cannon with exactly one
    screen, the facing generals rule, and a quiet rook move."""
    assert _check_bit("3k5/9/9/9/9/R8/9/9/9/4K4 w", 45, 48) == 1
    assert _check_bit("3k5/9/9/9/9/R8/9/9/9/4K4 w", 45, 46) == 0
    assert _check_bit("3k5/3p5/9/9/9/C8/9/9/9/4K4 w", 45, 48) == 1
    assert _check_bit("3k5/9/9/9/9/9/9/9/9/4K4 w", 85, 84) == 1
    # discovered: moving the screen away from a rook's file
    assert _check_bit("3k5/9/9/9/3P5/9/9/3R5/9/4K4 w", 39, 40) == 1


def test_policy_move_records_match_oracle():
    rng = np.random.default_rng(2)
    boards = az.random_boards(200, seed=21)
    n = 0
    for b in boards:
        for side in (0, 1):
            mv = az.pseudo_moves(b, side, rng, 25)
            if len(mv) == 0:
                continue
            np.testing.assert_array_equal(az.policy_moves(b, side, mv), oracle.az_policy_moves(b, side, mv))
            n += len(mv)
    assert n > 5000
