"""AZ-NNUE training: samples, the native batch packer, and the training step.

`pack_batch` takes the role of PackedBatch::from_indices
(src/az/dataloader.rs:113-336) through the C ABI (cnnue_az_pack_batch,
multi-threaded C++); `AzTrainer` that of GpuTrainer
(src/az/train_gpu_candle.rs:15-160): AzCandleModel::forward
(src/az/candle_model.rs:46-147) composed from this package's CUDA ops
(feature_pool, sparse_pool, fused_policy, sparse_policy, tactical_policy)
and dense cuBLAS matmuls, the loss of compute_batch_loss
(src/az/train_gpu_candle.rs:221-305), autograd, and the AdamW step of
candle-nn (lr, betas 0.9 / 0.999, eps 1e-8, weight decay 1e-4) as one CUDA
kernel over a flat parameter buffer.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields
from typing import Optional

import numpy as np

from . import az
from ._lib import check, lib

DENSE_MOVES = 2086
RULE_CONTEXT = 7
POLICY_MASK_VALUE = -1.0e9
SPARSE_TABLE = 2396815
SPARSE_FACTOR = 199458
TACTICAL = 934976


@dataclass
class Samples:
    """Training samples in CSR form (the AzTrainingSample fields the packer
    reads): canonical side-to-move features per sample, move indices with
    their policy targets, WDL / value targets, rule context, loss weights, ply."""
    features: np.ndarray         # u16 [total]
    feature_offsets: np.ndarray  # u32 [n + 1]
    move_indices: np.ndarray     # u16 [total moves]
    policy: np.ndarray           # f32 [total moves]
    move_offsets: np.ndarray     # u32 [n + 1]
    value_wdl: np.ndarray        # f32 [n, 3]
    value: np.ndarray            # f32 [n]
    rule_context: np.ndarray     # f32 [n, 7]
    policy_weight: np.ndarray    # f32 [n]
    value_weight: np.ndarray     # f32 [n]
    ply: np.ndarray              # u32 [n]

    @property
    def n(self) -> int:
        return len(self.feature_offsets) - 1


def random_samples(n: int, seed: int, max_moves: int = 40) -> Samples:
    """Synthetic samples of the self-play format: random boards (az.random_boards),
    a random side to move, its canonical features in board-scan order, up to
    `max_moves` pseudo moves in the dense space with gamma-distributed visit
    targets, random WDL / value / rule context / weights / ply.  A few samples
    carry the cases the packer must handle: features >= 1260, move indices
    >= 2086, moves whose source square holds no own piece, negative targets
    and weights, all-zero WDL, out-of-range values."""
    rng = np.random.default_rng(seed)
    boards = az.random_boards(n, seed ^ 0x5EED)
    _, s2d = az.dense_moves()
    feats, foff, moves, pol, moff = [], [0], [], [], [0]
    for i in range(n):
        side = int(rng.integers(0, 2))
        f = (az.features(boards[i], side) & 0x7FF).astype(np.uint16)
        if rng.random() < 0.05:
            f = np.append(f, np.uint16(1260 + rng.integers(0, 100)))
        feats.append(f)
        foff.append(foff[-1] + len(f))
        mv = az.pseudo_moves(boards[i], side, rng, int(rng.integers(1, max_moves + 1)))
        cf = mv[:, 0].astype(np.int64) if side == 0 else 89 - mv[:, 0].astype(np.int64)
        ct = mv[:, 1].astype(np.int64) if side == 0 else 89 - mv[:, 1].astype(np.int64)
        dense = s2d[cf * 90 + ct].astype(np.uint16)
        if rng.random() < 0.1:
            dense = np.append(dense, np.uint16(rng.integers(0, DENSE_MOVES)))  # any move, maybe no own piece
        if rng.random() < 0.05:
            dense = np.append(dense, np.uint16(DENSE_MOVES + rng.integers(0, 50)))  # outside the move space
        p = rng.gamma(0.5, 1.0, size=len(dense)).astype(np.float32)
        if rng.random() < 0.05:
            p[:] = 0.0
        if rng.random() < 0.05 and len(p):
            p[0] = -0.5
        moves.append(dense)
        pol.append(p)
        moff.append(moff[-1] + len(dense))
    wdl = rng.dirichlet([1.0, 1.0, 1.0], size=n).astype(np.float32)
    wdl[rng.random(n) < 0.03] = 0.0
    return Samples(
        features=np.concatenate(feats).astype(np.uint16) if feats else np.zeros(0, np.uint16),
        feature_offsets=np.array(foff, np.uint32),
        move_indices=np.concatenate(moves).astype(np.uint16) if moves else np.zeros(0, np.uint16),
        policy=np.concatenate(pol).astype(np.float32) if pol else np.zeros(0, np.float32),
        move_offsets=np.array(moff, np.uint32),
        value_wdl=wdl,
        value=rng.uniform(-1.2, 1.2, size=n).astype(np.float32),
        rule_context=rng.standard_normal((n, RULE_CONTEXT)).astype(np.float32),
        policy_weight=rng.uniform(-0.1, 1.5, size=n).astype(np.float32),
        value_weight=rng.uniform(-0.1, 1.5, size=n).astype(np.float32),
        ply=rng.integers(0, 200, size=n).astype(np.uint32),
    )


class _CSamples(C.Structure):
    _fields_ = [("n", C.c_int64)] + [(name, C.c_void_p) for name in (
        "features", "feature_offsets", "move_indices", "policy", "move_offsets", "value_wdl", "value",
        "rule_context", "policy_weight", "value_weight", "ply")]


@dataclass
class PackedBatch:
    """PackedBatch (src/az/dataloader.rs:92-111) as numpy arrays."""
    feature_items: np.ndarray           # u32 [B, F]
    value_threat_indices: np.ndarray    # u32 [B, T]
    policy_items: np.ndarray            # i64 [B, M]
    policy_sparse_indices: np.ndarray   # i64 [B, M, 7]
    policy_tactical_indices: np.ndarray  # i64 [B, M, 2]
    policy_targets: np.ndarray          # f32 [B, M]
    policy_mask: np.ndarray             # f32 [B, M]
    value_wdl: np.ndarray               # f32 [B, 3]
    values: np.ndarray                  # f32 [B]
    rule_context: np.ndarray            # f32 [B, 7]
    policy_weights: np.ndarray          # f32 [B]
    value_weights: np.ndarray           # f32 [B]
    value_phase_masks: np.ndarray       # f32 [B, 3]

    @property
    def batch_size(self) -> int:
        return self.values.shape[0]


_PACKED_FIELDS = [f.name for f in fields(PackedBatch)]


class _CPacked(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("batch", "max_features", "max_policy_moves", "max_value_threats")] + \
        [(name, C.c_void_p) for name in _PACKED_FIELDS]


def _samples_struct(s: Samples, keep: list) -> _CSamples:
    arrays = [np.ascontiguousarray(a, dt) for a, dt in (
        (s.features, np.uint16), (s.feature_offsets, np.uint32), (s.move_indices, np.uint16),
        (s.policy, np.float32), (s.move_offsets, np.uint32), (s.value_wdl, np.float32), (s.value, np.float32),
        (s.rule_context, np.float32), (s.policy_weight, np.float32), (s.value_weight, np.float32),
        (s.ply, np.uint32))]
    arrays = [a if a.size else np.zeros(1, a.dtype) for a in arrays]
    keep.extend(arrays)
    return _CSamples(s.n, *[a.ctypes.data for a in arrays])


def pack_batch(samples: Samples, rows: Optional[np.ndarray] = None, n_threads: int = 0,
               caps=(96, 160, 256)) -> PackedBatch:
    """Packs samples[rows] (all samples when rows is None) with the native packer."""
    keep: list = []
    cs = _samples_struct(samples, keep)
    if rows is None:
        batch, rptr = samples.n, None
    else:
        r = np.ascontiguousarray(rows, np.int64)
        keep.append(r)
        batch, rptr = len(r), (r.ctypes.data if len(r) else None)
    while True:
        F, M, T = caps
        b = max(batch, 1)
        bufs = {
            "feature_items": np.empty((b, F), np.uint32), "value_threat_indices": np.empty((b, T), np.uint32),
            "policy_items": np.empty((b, M), np.int64), "policy_sparse_indices": np.empty((b, M, 7), np.int64),
            "policy_tactical_indices": np.empty((b, M, 2), np.int64), "policy_targets": np.empty((b, M), np.float32),
            "policy_mask": np.empty((b, M), np.float32), "value_wdl": np.empty((b, 3), np.float32),
            "values": np.empty(b, np.float32), "rule_context": np.empty((b, RULE_CONTEXT), np.float32),
            "policy_weights": np.empty(b, np.float32), "value_weights": np.empty(b, np.float32),
            "value_phase_masks": np.empty((b, 3), np.float32)}
        out = _CPacked(0, 0, 0, 0, *[bufs[k].ctypes.data for k in _PACKED_FIELDS])
        st = lib().cnnue_az_pack_batch(C.byref(cs), rptr, batch, F, M, T, C.byref(out), n_threads)
        need = (out.max_features, out.max_policy_moves, out.max_value_threats)
        if st == 5 and any(n > c for n, c in zip(need, caps)):  # CNNUE_ERR_WORKSPACE: grow and retry
            caps = tuple(max(n, c) for n, c in zip(need, caps))
            continue
        check(st, "cnnue_az_pack_batch")
        break
    F, M, T = need

    def cut(a, width, extra=()):
        flat = a.reshape(-1)[: batch * width * int(np.prod(extra or (1,)))]
        return flat.reshape((batch, width) + tuple(extra))

    return PackedBatch(
        feature_items=cut(bufs["feature_items"], F), value_threat_indices=cut(bufs["value_threat_indices"], T),
        policy_items=cut(bufs["policy_items"], M), policy_sparse_indices=cut(bufs["policy_sparse_indices"], M, (7,)),
        policy_tactical_indices=cut(bufs["policy_tactical_indices"], M, (2,)),
        policy_targets=cut(bufs["policy_targets"], M), policy_mask=cut(bufs["policy_mask"], M),
        value_wdl=bufs["value_wdl"][:batch], values=bufs["values"][:batch],
        rule_context=bufs["rule_context"][:batch], policy_weights=bufs["policy_weights"][:batch],
        value_weights=bufs["value_weights"][:batch], value_phase_masks=bufs["value_phase_masks"][:batch])
