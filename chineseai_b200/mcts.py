"""Wide-batch AlphaZero search over the GPU evaluator (cnnue_mcts_* of the C
ABI): many roots searched in lockstep, one GPU batch of leaves per round.

Takes the role of the reference's batch-of-four search
(alphazero_search_batch4_reusing, src/az/alphazero.rs:388-521) and of AzTree's
PUCT selection, expansion and backup; `legal_moves` that of
Position::legal_moves (src/xiangqi/mod.rs) without the repetition rules.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from ._lib import check, lib


class Limits(C.Structure):
    """AzSearchLimits (src/az/alphazero.rs:22-66) less seed and root noise."""
    _fields_ = [("simulations", C.c_int64)] + \
        [(n, C.c_float) for n in ("cpuct", "cpuct_at_root", "cpuct_base", "cpuct_factor", "cpuct_base_at_root",
                                  "cpuct_factor_at_root")] + \
        [("max_depth", C.c_int64)] + \
        [(n, C.c_float) for n in ("fpu_value", "fpu_value_at_root", "policy_softmax_temp", "draw_score",
                                  "value_scale")]


def default_limits(simulations: Optional[int] = None) -> Limits:
    lim = Limits()
    lib().cnnue_mcts_default_limits(C.byref(lim))
    if simulations is not None:
        lim.simulations = simulations
    return lim


def legal_moves(board: np.ndarray, side: int) -> np.ndarray:
    """Legal moves of `side` as uint8 [n][2] (from, to) squares."""
    b = np.ascontiguousarray(board, np.int8)
    out = np.zeros((128, 2), np.uint8)
    n = C.c_int()
    check(lib().cnnue_az_legal_moves(b.ctypes.data, side, out.ctypes.data, 128, C.byref(n)), "cnnue_az_legal_moves")
    return out[:n.value].copy()


def perft(board: np.ndarray, side: int, depth: int) -> int:
    """Leaf count of the legal-move tree (moves applied without rules history)."""
    if depth == 0:
        return 1
    moves = legal_moves(board, side)
    if depth == 1:
        return len(moves)
    total = 0
    for frm, to in moves:
        child = board.copy()
        child[to] = child[frm]
        child[frm] = 0
        total += perft(child, 1 - side, depth - 1)
    return total


class Search:
    """cnnue_mcts over an AzModel (device evaluator) and its AzWeights."""

    def __init__(self, model, weights, n_threads: int = 0):
        self._h = C.c_void_p()
        check(lib().cnnue_mcts_create(model.handle, weights.handle, n_threads, C.byref(self._h)),
              "cnnue_mcts_create")
        self._keep = (model, weights)
        self.n_roots = 0

    def run(self, boards: np.ndarray, sides: np.ndarray, limits: Limits,
            rule_context: Optional[np.ndarray] = None, stream=None) -> int:
        """Searches every root; returns the number of network evaluations."""
        b = np.ascontiguousarray(boards, np.int8).reshape(-1, 90)
        s = np.ascontiguousarray(sides, np.uint8).reshape(-1)
        r = None if rule_context is None else np.ascontiguousarray(rule_context, np.float32).reshape(-1, 7)
        evals = C.c_uint64()
        st = 0 if stream is None else stream
        check(lib().cnnue_mcts_search(self._h, b.ctypes.data, s.ctypes.data, None if r is None else r.ctypes.data,
                                      len(b), C.byref(limits), st, C.byref(evals)), "cnnue_mcts_search")
        self.n_roots = len(b)
        return evals.value

    def stats(self) -> dict:
        """Seconds of the last search by phase and its number of GPU rounds."""
        sec = np.zeros(4, np.float64)
        rounds = C.c_uint64()
        check(lib().cnnue_mcts_stats(self._h, sec.ctypes.data, C.byref(rounds)), "cnnue_mcts_stats")
        return {"select_s": sec[0], "inputs_s": sec[1], "gpu_s": sec[2], "finalize_s": sec[3],
                "rounds": rounds.value}

    def result(self, root: int) -> dict:
        cap = 128
        moves = np.zeros((cap, 2), np.uint8)
        visits = np.zeros(cap, np.uint32)
        priors = np.zeros(cap, np.float32)
        q = np.zeros(cap, np.float32)
        n, best = C.c_int(), C.c_int()
        root_q, root_visits = C.c_float(), C.c_uint32()
        check(lib().cnnue_mcts_result(self._h, root, moves.ctypes.data, visits.ctypes.data, priors.ctypes.data,
                                      q.ctypes.data, cap, C.byref(n), C.byref(best), C.byref(root_q),
                                      C.byref(root_visits)), "cnnue_mcts_result")
        k = n.value
        return {"moves": moves[:k].copy(), "visits": visits[:k].copy(), "priors": priors[:k].copy(),
                "q": q[:k].copy(), "best": best.value, "root_q": root_q.value, "root_visits": root_visits.value}

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_mcts_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
