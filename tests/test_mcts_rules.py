"""Move generation of the wide-batch search: the published perft counts of
the xiangqi start position (44, 1,920, 79,666, 3,290,240), and equality - the
same moves in the same order, the order the search's forced replies and ties
depend on - with the oracle's independent Python restatement of the move
rules on random boards, both sides, including positions in check."""
import numpy as np
import pytest

from chineseai_b200 import az, mcts
from oracle import mcts_ref

START = "rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR w - - 0 1"


@pytest.mark.parametrize("depth,count", [(1, 44), (2, 1920), (3, 79666), (4, 3290240)])
def test_start_position_perft(depth, count):
    b, side = az.board_from_fen(START)
    assert mcts.perft(b, side, depth) == count


def test_black_start_moves_and_python_restatement():
    b, _ = az.board_from_fen(START)
    assert len(mcts.legal_moves(b, 1)) == 44
    assert sorted(map(tuple, mcts.legal_moves(b, 0).tolist())) == sorted(mcts_ref.legal_moves(b, 0))


def test_random_boards_match_restatement():
    boards = az.random_boards(300, seed=5, keep=0.7)
    checks = 0
    for i, b in enumerate(boards):
        for side in (0, 1):
            got = list(map(tuple, mcts.legal_moves(b, side).tolist()))
            want = mcts_ref.legal_moves(b, side)
            assert got == want, (i, side)  # same moves in the same order
            checks += mcts_ref.in_check(b, side)
    assert checks > 0  # positions in check were covered


def test_facing_generals_and_pins():
    b = np.zeros(90, np.int8)
    b[4] = -1            # Black general e10 (rank 0, file 4)
    b[85] = 1            # Red general e1 (rank 9, file 4)
    b[49] = 5            # Red rook on the e-file between them: pinned to the file
    moves = mcts.legal_moves(b, 0)
    rook = [tuple(m) for m in moves.tolist() if m[0] == 49]
    assert rook and all(to % 9 == 4 for _, to in rook)
    # the Red general may not step onto the open file facing the Black general: nothing blocks after 49 leaves
    assert sorted(map(tuple, moves.tolist())) == sorted(mcts_ref.legal_moves(b, 0))


def test_playout_positions_match_restatement():
    """Positions from random legal playouts of 1-80 plies from the start (the
    search's own inputs: checks, pins of every kind, cannon screens, horse
    legs next to the general), both sides to move: the same legal moves in
    the same order.  Guards the generator's shortcut that skips the attack
    test for moves that cannot expose the general."""
    rng = np.random.default_rng(11)
    b0, s0 = az.board_from_fen(START)
    n, checks = 0, 0
    while n < 1000:
        b, side = b0.copy(), s0
        for _ in range(int(rng.integers(1, 81))):
            moves = mcts.legal_moves(b, side)  # fast; the end positions are compared below
            if not len(moves) or not (b == -1).any() or not (b == 1).any():
                break
            frm, to = moves[rng.integers(len(moves))]
            b[to], b[frm] = b[frm], 0
            side = 1 - side
        for s in (0, 1):
            got = list(map(tuple, mcts.legal_moves(b, s).tolist()))
            assert got == mcts_ref.legal_moves(b, s), (n, s)
            checks += mcts_ref.in_check(b, s)
        n += 1
    assert checks > 10
