"""Host-side API of the reference-native AZ-NNUE evaluator (over the C ABI).

Mirrors the reference's `AzNnue` (src/az.rs:861-901) for its trunk and value
head:

* `AzWeights` - the 22 fp32 tensors of `az_weight_tensors!` (src/az.rs:241-278):
  `AzWeights.random(hidden, seed)` is `AzNnue::random` (src/az.rs:1433-1435,
  :1339-1431), `load` / `save` read and write the reference's safetensors file
  (src/az.rs:1437-1529).  Tensors are numpy views of the library's host copy.
* `AzModel` - the device-resident trunk and value head on one GPU:
  `refresh` (AzEvalAccumulator::refresh, src/az.rs:384-411), `transition`
  (apply_transition_for_perspective, src/az.rs:439-485) and `value`
  (the value part of evaluate_incremental_with_scratch_output,
  src/az.rs:1606-1652).
* `board_from_fen`, `features`, `move_items` - the host steps the reference
  does inside those calls (src/xiangqi/mod.rs:163-207, src/nnue.rs:31-43).

Device buffers are torch CUDA tensors; every computation runs in libcnnue's
kernels, and a missing library raises at import of `_lib.lib()`.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np

from ._lib import check, lib

SQUARES = 90
INPUT = 1260
TRUNK_ROWS = 1545
VALUE_HEAD = 96
RULE_CONTEXT = 7
N_TENSORS = 22
NO_ITEM = 0xFFFFFFFF
FORMAT_VERSION = 20.0
STARTPOS = "rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR w"

# Quantised tables (cnnue_az_quant_table).
Q_POLICY_FEATURE, Q_POLICY_MOVE, Q_POLICY_SPARSE, Q_VALUE_THREAT, Q_MOVED_DELTA, Q_CAPTURE = range(6)
DENSE_MOVES = 2086


def dense_moves() -> Tuple[np.ndarray, np.ndarray]:
    """(dense_to_sparse uint16[2086], sparse_to_dense uint16[8100])."""
    d2s = np.zeros(DENSE_MOVES, np.uint16)
    s2d = np.zeros(SQUARES * SQUARES, np.uint16)
    check(lib().cnnue_az_dense_moves(d2s.ctypes.data, s2d.ctypes.data), "cnnue_az_dense_moves")
    return d2s, s2d


# Piece codes of a board: +(kind+1) Red, -(kind+1) Black.
GENERAL, ADVISOR, ELEPHANT, HORSE, ROOK, CANNON, SOLDIER = range(7)


def tensor_info(index: int, hidden: int) -> Tuple[str, int]:
    name = C.c_char_p()
    count = C.c_int64()
    check(lib().cnnue_az_tensor_info(index, hidden, C.byref(name), C.byref(count)), "cnnue_az_tensor_info")
    return name.value.decode(), count.value


def tensor_shape(index: int, hidden: int) -> Tuple[int, ...]:
    """Shape of tensor `index` as az_weight_tensors! declares it."""
    rows = {0: 1260, 1: 14, 2: 10, 3: 9, 4: 252, 5: 7, 7: 96, 9: 3, 10: 57702, 11: 3, 12: 16, 15: 16, 16: 2086,
            17: 32, 18: 2086}
    _, count = tensor_info(index, hidden)
    if index in rows:
        return rows[index], count // rows[index]
    return (count,)


class AzWeights:
    """Host copy of the AZ-NNUE weights (owned by libcnnue)."""

    def __init__(self, handle: C.c_void_p):
        self._h = handle
        self.hidden = int(lib().cnnue_az_weights_hidden(handle))
        self.names: List[str] = [tensor_info(i, self.hidden)[0] for i in range(N_TENSORS)]

    @classmethod
    def random(cls, hidden: int = 128, seed: int = 20260807) -> "AzWeights":
        h = C.c_void_p()
        check(lib().cnnue_az_weights_random(hidden, seed, C.byref(h)), "cnnue_az_weights_random")
        return cls(h)

    @classmethod
    def load(cls, path: str) -> "AzWeights":
        h = C.c_void_p()
        check(lib().cnnue_az_weights_load(str(path).encode(), C.byref(h)), "cnnue_az_weights_load")
        return cls(h)

    def save(self, path: str) -> None:
        check(lib().cnnue_az_weights_save(self._h, str(path).encode()), "cnnue_az_weights_save")

    def tensor(self, index_or_name) -> np.ndarray:
        """Writable numpy view (shape as declared) of one tensor."""
        index = self.names.index(index_or_name) if isinstance(index_or_name, str) else int(index_or_name)
        ptr = C.POINTER(C.c_float)()
        count = C.c_int64()
        check(lib().cnnue_az_weights_tensor(self._h, index, C.byref(ptr), C.byref(count)), "cnnue_az_weights_tensor")
        flat = np.ctypeslib.as_array(ptr, shape=(count.value,)) if count.value else np.zeros(0, np.float32)
        return flat.reshape(tensor_shape(index, self.hidden))

    def tensors(self) -> List[np.ndarray]:
        return [self.tensor(i) for i in range(N_TENSORS)]

    def quantize(self) -> None:
        """Rebuilds the quantised tables after tensor edits (the reference's
        rebuild_* steps, src/az.rs:2201-2342)."""
        check(lib().cnnue_az_quantize(self._h), "cnnue_az_quantize")

    def quant_table(self, which: int) -> Tuple[np.ndarray, float]:
        """(copy of quantised table `which` (Q_*), its scale)."""
        data = C.c_void_p()
        count = C.c_int64()
        scale = C.c_float()
        check(lib().cnnue_az_quant_table(self._h, which, C.byref(data), C.byref(count), C.byref(scale)),
              "cnnue_az_quant_table")
        ctype, dtype = (C.c_int8, np.int8) if which < 4 else (C.c_int32, np.int32)
        arr = np.ctypeslib.as_array(C.cast(data, C.POINTER(ctype)), shape=(count.value,)).astype(dtype)
        shapes = {Q_POLICY_FEATURE: (1546, 32), Q_POLICY_MOVE: (2086, 32), Q_VALUE_THREAT: (57702, 64),
                  Q_MOVED_DELTA: (2086, 14), Q_CAPTURE: (2086, 14)}
        return arr.reshape(shapes.get(which, (count.value,))), scale.value

    def quant_flags(self) -> Tuple[bool, bool]:
        """(value_threat_active, policy_tactical_active)."""
        a, b = C.c_int(), C.c_int()
        check(lib().cnnue_az_quant_flags(self._h, C.byref(a), C.byref(b)), "cnnue_az_quant_flags")
        return bool(a.value), bool(b.value)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_az_weights_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- boards -----------------------------------------------------------------
def board_from_fen(fen: str) -> Tuple[np.ndarray, int]:
    board = np.zeros(SQUARES, np.int8)
    side = C.c_int()
    check(lib().cnnue_az_board_from_fen(fen.encode(), board.ctypes.data, C.byref(side)), "cnnue_az_board_from_fen")
    return board, side.value


def features(board: np.ndarray, perspective: int) -> np.ndarray:
    """Packed items (feature | us << 11 | them << 15) in board-scan order."""
    b = np.ascontiguousarray(board, np.int8)
    items = np.zeros(SQUARES, np.uint32)
    n = C.c_int()
    check(lib().cnnue_az_features(b.ctypes.data, perspective, items.ctypes.data, C.byref(n)), "cnnue_az_features")
    return items[:n.value].copy()


THREAT_VOCAB = 57702
THREAT_MAX = 256


def threat_features(board: np.ndarray, side: int) -> np.ndarray:
    """Threat-table rows of the side to move (value_threat_index of every
    attack on an occupied square, source-square order)."""
    b = np.ascontiguousarray(board, np.int8)
    out = np.zeros(THREAT_MAX, np.uint32)
    n = C.c_int()
    check(lib().cnnue_az_threat_features(b.ctypes.data, side, out.ctypes.data, C.byref(n)),
          "cnnue_az_threat_features")
    return out[:n.value].copy()


def policy_moves(board: np.ndarray, side: int, moves: np.ndarray) -> np.ndarray:
    """Per-move records uint32 [n][2] for the policy logits (moves: [n][2]
    absolute from/to squares)."""
    b = np.ascontiguousarray(board, np.int8)
    mv = np.ascontiguousarray(moves, np.uint8).reshape(-1, 2)
    info = np.zeros((max(len(mv), 1), 2), np.uint32)
    check(lib().cnnue_az_policy_moves(b.ctypes.data, side, mv.ctypes.data, len(mv), info.ctypes.data),
          "cnnue_az_policy_moves")
    return info[:len(mv)].copy()


def pseudo_moves(board: np.ndarray, side: int, rng: np.random.Generator, k: int) -> np.ndarray:
    """Up to k distinct from/to pairs of `side`'s pieces onto empty or enemy
    squares that lie in the dense policy move space (stand-ins for a move
    list; rules legality is not needed by the arithmetic)."""
    _, s2d = dense_moves()
    own = np.flatnonzero((board > 0) if side == 0 else (board < 0))
    out = []
    for _ in range(8 * k):
        if len(out) == k or len(own) == 0:
            break
        frm = int(rng.choice(own))
        to = int(rng.integers(0, SQUARES))
        if to == frm or (board[to] != 0 and (board[to] > 0) == (board[frm] > 0)):
            continue
        cf, ct = (frm, to) if side == 0 else (89 - frm, 89 - to)
        if s2d[cf * SQUARES + ct] == 0xFFFF or (frm, to) in out:
            continue
        out.append((frm, to))
    return np.array(out, np.uint8).reshape(-1, 2)


@dataclass
class MoveItems:
    refresh: bool
    delta: np.ndarray  # uint32[3]: from, captured (or NO_ITEM), to
    items: np.ndarray  # the child's items when refresh


def move_items(board: np.ndarray, frm: int, to: int, perspective: int) -> MoveItems:
    b = np.ascontiguousarray(board, np.int8)
    delta = np.zeros(3, np.uint32)
    refresh = np.zeros(1, np.uint8)
    items = np.zeros(SQUARES, np.uint32)
    n = C.c_int()
    check(lib().cnnue_az_move_items(b.ctypes.data, frm, to, perspective, delta.ctypes.data, refresh.ctypes.data,
                                    items.ctypes.data, C.byref(n)), "cnnue_az_move_items")
    return MoveItems(bool(refresh[0]), delta, items[:n.value].copy())


def apply_move(board: np.ndarray, frm: int, to: int) -> np.ndarray:
    after = board.copy()
    after[to] = after[frm]
    after[frm] = 0
    return after


# Standard material of one side: general, 2 advisors, 2 elephants, 2 horses,
# 2 rooks, 2 cannons, 5 soldiers.
_MATERIAL = [GENERAL] + [ADVISOR] * 2 + [ELEPHANT] * 2 + [HORSE] * 2 + [ROOK] * 2 + [CANNON] * 2 + [SOLDIER] * 5


def random_boards(n: int, seed: int, keep: float = 0.85, generals: bool = True) -> np.ndarray:
    """n synthetic boards int8[n][90]: each general on a random square of its
    palace (Red ranks 7-9, Black ranks 0-2, files 3-5), every other piece of the
    standard material kept with probability `keep` on a random empty square."""
    rng = np.random.default_rng(seed)
    boards = np.zeros((n, SQUARES), np.int8)
    for i in range(n):
        b = boards[i]
        for color, sign, ranks in ((0, 1, (7, 8, 9)), (1, -1, (0, 1, 2))):
            if generals:
                b[int(rng.choice(ranks)) * 9 + int(rng.integers(3, 6))] = sign * (GENERAL + 1)
            for kind in _MATERIAL[1:]:
                if rng.random() >= keep:
                    continue
                empty = np.flatnonzero(b == 0)
                b[int(rng.choice(empty))] = sign * (kind + 1)
    return boards


def random_move(board: np.ndarray, rng: np.random.Generator, side: Optional[int] = None) -> Tuple[int, int]:
    """A random from -> to of a piece (of `side` if given) onto an empty or
    enemy square; not a rules-legal move, but the same accumulator arithmetic."""
    occupied = np.flatnonzero(board != 0)
    if side is not None:
        occupied = occupied[(board[occupied] > 0) == (side == 0)]
    frm = int(rng.choice(occupied))
    mine = board[frm] > 0
    targets = np.flatnonzero((board == 0) | ((board > 0) != mine))
    return frm, int(rng.choice(targets))


def pack_lists(lists: Sequence[np.ndarray]) -> Tuple[np.ndarray, np.ndarray]:
    """CSR packing: (items uint32[total], offsets uint32[len+1])."""
    offsets = np.zeros(len(lists) + 1, np.uint32)
    if lists:
        offsets[1:] = np.cumsum([len(x) for x in lists])
    items = np.concatenate(lists).astype(np.uint32) if lists and offsets[-1] else np.zeros(0, np.uint32)
    return items, offsets


def node_lists(boards: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Items of both perspectives of every board: list 2i = Red, 2i+1 = Black
    (the [2][H] node accumulator of AzEvalAccumulator)."""
    return pack_lists([features(b, p) for b in boards for p in (0, 1)])


# ---- device model -----------------------------------------------------------
class AzModel:
    """Trunk + value head of an AzNnue on one GPU (hidden <= 512)."""

    def __init__(self, weights: AzWeights, device: int = 0):
        import torch
        self._torch = torch
        self.device = torch.device("cuda", device)
        self.hidden = weights.hidden
        h = C.c_void_p()
        check(lib().cnnue_az_model_create(weights.handle, device, C.byref(h)), "cnnue_az_model_create")
        self._h = h
        self._ws = torch.zeros(int(lib().cnnue_az_workspace_bytes()), dtype=torch.uint8, device=self.device)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def workspace(self):
        return self._ws

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_az_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self, stream) -> int:
        s = stream if stream is not None else self._torch.cuda.current_stream(self.device)
        return s.cuda_stream

    def read_status(self, stream=None) -> int:
        st = C.c_int(0)
        check(lib().cnnue_read_status(self._ws.data_ptr(), self._stream(stream), C.byref(st)), "cnnue_read_status")
        return st.value

    @staticmethod
    def _ptr(t) -> Optional[int]:
        return None if t is None else t.data_ptr()

    def refresh(self, items, offsets, out=None, stream=None):
        """acc [n_lists][H] from CSR item lists (device uint32/int32 tensors)."""
        torch = self._torch
        n_lists = offsets.numel() - 1
        if out is None:
            out = torch.empty((n_lists, self.hidden), dtype=torch.float32, device=self.device)
        check(lib().cnnue_az_refresh(self._h, self._ptr(items) if items.numel() else None, items.numel(),
                                     offsets.data_ptr(), n_lists, out.data_ptr(), self._ws.data_ptr(),
                                     self._ws.numel(), self._stream(stream)), "cnnue_az_refresh")
        return out

    def transition(self, parent, delta, refresh, items=None, offsets=None, out=None, stream=None):
        """child [n_lists][H]: parent -/+ the delta rows, or a refresh of the
        list where refresh[l] is set.  out may be parent (in place)."""
        torch = self._torch
        n_lists = refresh.numel()
        if out is None:
            out = torch.empty((n_lists, self.hidden), dtype=torch.float32, device=self.device)
        n_items = 0 if items is None else items.numel()
        check(lib().cnnue_az_transition(self._h, parent.data_ptr(), delta.data_ptr(), refresh.data_ptr(),
                                        self._ptr(items) if n_items else None, n_items, self._ptr(offsets),
                                        n_lists, out.data_ptr(), self._ws.data_ptr(), self._ws.numel(),
                                        self._stream(stream)), "cnnue_az_transition")
        return out

    def policy_refresh(self, items, offsets, out=None, stream=None):
        """int16 policy accumulators [n_lists][32] from CSR item lists."""
        torch = self._torch
        n_lists = offsets.numel() - 1
        if out is None:
            out = torch.empty((n_lists, 32), dtype=torch.int16, device=self.device)
        check(lib().cnnue_az_policy_refresh(self._h, self._ptr(items) if items.numel() else None, items.numel(),
                                            offsets.data_ptr(), n_lists, out.data_ptr(), self._ws.data_ptr(),
                                            self._ws.numel(), self._stream(stream)), "cnnue_az_policy_refresh")
        return out

    def policy_transition(self, parent, delta, refresh, items=None, offsets=None, out=None, stream=None):
        torch = self._torch
        n_lists = refresh.numel()
        if out is None:
            out = torch.empty((n_lists, 32), dtype=torch.int16, device=self.device)
        n_items = 0 if items is None else items.numel()
        check(lib().cnnue_az_policy_transition(self._h, parent.data_ptr(), delta.data_ptr(), refresh.data_ptr(),
                                               self._ptr(items) if n_items else None, n_items, self._ptr(offsets),
                                               n_lists, out.data_ptr(), self._ws.data_ptr(), self._ws.numel(),
                                               self._stream(stream)), "cnnue_az_policy_transition")
        return out

    def threat_logits(self, features, offsets, out=None, stream=None):
        """Threat logits [n][3] from CSR threat features (device uint32)."""
        torch = self._torch
        n = offsets.numel() - 1
        if out is None:
            out = torch.empty((n, 3), dtype=torch.float32, device=self.device)
        check(lib().cnnue_az_threat_logits(self._h, self._ptr(features) if features.numel() else None,
                                           features.numel(), offsets.data_ptr(), n, out.data_ptr(),
                                           self._ws.data_ptr(), self._ws.numel(), self._stream(stream)),
              "cnnue_az_threat_logits")
        return out

    def evaluate(self, acc, side=None, rule=None, threat_features=None, threat_offsets=None, policy_acc=None,
                 move_info=None, move_offsets=None, stream=None):
        """evaluate_incremental_with_scratch_output for a batch: (wdl, q,
        logits or None).  acc/policy_acc are node layouts with `side`."""
        torch = self._torch
        n = side.numel() if side is not None else acc.numel() // self.hidden
        wdl = torch.empty((n, 3), dtype=torch.float32, device=self.device)
        q = torch.empty(n, dtype=torch.float32, device=self.device)
        logits = None
        n_moves = 0
        if move_info is not None:
            n_moves = move_info.numel() // 2
            logits = torch.empty(n_moves, dtype=torch.float32, device=self.device)
        need = int(lib().cnnue_az_evaluate_workspace_bytes(self._h, n))
        if self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        n_tf = 0 if threat_features is None else threat_features.numel()
        check(lib().cnnue_az_evaluate(self._h, acc.data_ptr(), self._ptr(side), self._ptr(rule),
                                      self._ptr(threat_features) if n_tf else None, n_tf, self._ptr(threat_offsets),
                                      self._ptr(policy_acc), self._ptr(move_info), n_moves, self._ptr(move_offsets),
                                      n, wdl.data_ptr(), q.data_ptr(), self._ptr(logits), self._ws.data_ptr(),
                                      self._ws.numel(), self._stream(stream)), "cnnue_az_evaluate")
        return wdl, q, logits

    def value(self, acc, side=None, rule=None, threat=None, stream=None):
        """(wdl [n][3], q [n]) of side-to-move accumulators: acc [n][H], or with
        `side` (uint8 [n], 0 Red) the node accumulators [n][2][H] / [2n][H]."""
        torch = self._torch
        n = acc.numel() // self.hidden if side is None else side.numel()
        if acc.numel() != n * self.hidden * (1 if side is None else 2):
            raise ValueError(f"acc has {acc.numel()} floats, expected {n} x {1 if side is None else 2} x {self.hidden}")
        wdl = torch.empty((n, 3), dtype=torch.float32, device=self.device)
        q = torch.empty(n, dtype=torch.float32, device=self.device)
        check(lib().cnnue_az_value(self._h, acc.data_ptr(), self._ptr(side), self._ptr(rule), self._ptr(threat), n,
                                   wdl.data_ptr(), q.data_ptr(), self._stream(stream)), "cnnue_az_value")
        return wdl, q
