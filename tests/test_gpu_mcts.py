"""The wide-batch GPU search against the oracle's restatement of AzTree (one
root at a time, leaves evaluated by the oracle's C evaluator): the same root
visit counts and best move, priors within the evaluator's 1e-4; deterministic
repeats; many roots in one batch; terminal and move-less roots."""
import numpy as np
import pytest

from chineseai_b200 import az, mcts
from oracle import mcts_ref
from tests._azutil import full_policy, trained_like

pytestmark = pytest.mark.gpu
START = "rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR w - - 0 1"


@pytest.fixture(scope="module")
def setup():
    w = az.AzWeights.random(128, 20260821)
    trained_like(w, 71)
    full_policy(w, 72)
    model = az.AzModel(w, device=0)
    yield w, model
    model.close()


def roots(n, seed):
    """The start position and positions after 1-40 random legal moves from it."""
    rng = np.random.default_rng(seed)
    b0, s0 = az.board_from_fen(START)
    boards, sides = [b0], [s0]
    while len(boards) < n:
        b, side = b0.copy(), s0
        for _ in range(int(rng.integers(1, 41))):
            moves = mcts.legal_moves(b, side)
            if len(moves) == 0 or not (b == -1).any() or not (b == 1).any():
                break
            frm, to = moves[rng.integers(len(moves))]
            b[to], b[frm] = b[frm], 0
            side = 1 - side
        if (b == -1).any() and (b == 1).any() and len(mcts.legal_moves(b, side)):
            boards.append(b)
            sides.append(side)
    return np.array(boards, np.int8), np.array(sides, np.uint8)


def test_matches_reference_search(setup):
    w, model = setup
    threat, tactical = w.quant_flags()
    assert threat and tactical
    boards, sides = roots(4, 3)
    sims = 48
    search = mcts.Search(model, w, n_threads=4)
    evals = search.run(boards, sides, mcts.default_limits(sims))
    assert evals > 0
    ev = mcts_ref.Evaluator(w.tensors(), 128, threat, tactical)
    for i in range(len(boards)):
        got = search.result(i)
        ref = mcts_ref.Search(ev, boards[i], int(sides[i]), sims).run().result()
        assert [tuple(m) for m in got["moves"].tolist()] == ref["moves"]
        np.testing.assert_allclose(got["priors"], ref["priors"], atol=1e-4)
        assert got["visits"].tolist() == ref["visits"], i
        assert got["root_visits"] == sims
        assert int(np.argmax(got["visits"])) == int(np.argmax(ref["visits"])) or \
            got["visits"][got["best"]] == max(got["visits"])


def test_deterministic_and_wide(setup):
    w, model = setup
    boards, sides = roots(300, 9)
    lim = mcts.default_limits(24)
    s1 = mcts.Search(model, w)
    e1 = s1.run(boards, sides, lim)
    r1 = [s1.result(i) for i in range(len(boards))]
    s2 = mcts.Search(model, w, n_threads=3)
    e2 = s2.run(boards, sides, lim)
    assert e1 == e2
    for i in range(len(boards)):
        r2 = s2.result(i)
        assert r1[i]["visits"].tolist() == r2["visits"].tolist()
        assert r1[i]["best"] == r2["best"] and r1[i]["root_visits"] == 24
    # the root expansions plus at least one leaf per simulation of most roots
    # (forced replies add leaves inside a simulation)
    assert e1 >= len(boards) * 20


def test_terminal_and_moveless_roots(setup):
    w, model = setup
    b, _ = az.board_from_fen(START)
    no_black_general = b.copy()
    no_black_general[no_black_general == -1] = 0
    # Black to move with its general in the corner of the palace, checked by a
    # rook and with both exits covered: no legal move, a loss for Black
    mated = np.zeros(90, np.int8)
    mated[3] = -1      # Black general d10
    mated[85] = 1      # Red general e1
    mated[12] = 5      # Red rook d9: checks the general, covers d10
    mated[14] = 5      # Red rook f9 (behind d9 along rank 9): protects d9 and covers e9
    assert len(mcts.legal_moves(mated, 1)) == 0
    boards = np.stack([no_black_general, mated, b])
    sides = np.array([0, 1, 0], np.uint8)
    search = mcts.Search(model, w)
    search.run(boards, sides, mcts.default_limits(8))
    r = search.result(0)
    assert len(r["moves"]) == 0 and r["root_visits"] == 8 and r["root_q"] > 0.99  # Red to move, Black lost
    r = search.result(1)
    assert len(r["moves"]) == 0 and r["root_visits"] == 8 and r["root_q"] < -0.99
    assert search.result(2)["root_visits"] == 8
