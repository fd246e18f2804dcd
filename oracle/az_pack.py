"""Training batch packer restated - TEST INFRASTRUCTURE ONLY.

PackedBatch::from_indices (src/az/dataloader.rs:113-336) in plain Python
loops over the oracle's C board helpers: threat features (value_threat_features,
:307-326, via oracle_az_threat_features) and the tactical signature bits
(attacked_squares_mask / gives_check_after_move_fast, via
oracle_az_policy_moves on the canonical position, Red to move).  Everything
else - buckets (src/az.rs:168-203), pack_feature, pack_policy_item
(src/az/fused_policy.rs:146-157), the sparse / factor / tactical indices
(src/az.rs:763-859), target normalisation (:432-446, src/az.rs:2586-2599) -
is restated here.  Used only to check the native packer.
"""
from __future__ import annotations

import numpy as np

from . import az_dense_moves, az_policy_moves, az_threat_features

F32 = np.float32
SPARSE_TABLE = 2396815
SPARSE_MAIN = 2086 * 14 * 81
TACTICAL_EXACT = 2086 * 7 * 64
TACTICAL = TACTICAL_EXACT + 7 * 64
PAD = 0xFFFFFFFF


def _general_bucket(piece_index, sq):
    o = sq if piece_index < 7 else 89 - sq
    f, r = min(max(o % 9, 3), 5), min(max(o // 9, 7), 9)
    return (r - 7) * 3 + (f - 3)


def _max0(x):
    """f32::max(x, 0.0): NaN gives 0."""
    return F32(0.0) if np.isnan(x) else max(F32(x), F32(0.0))


def pack(samples, rows=None):
    moves_map = az_dense_moves()
    rows = list(range(samples.n)) if rows is None else [int(r) for r in rows]
    per = []
    for i in rows:
        f = [int(x) for x in samples.features[samples.feature_offsets[i]:samples.feature_offsets[i + 1]]]
        board = np.zeros(90, np.int8)
        bf = [-1] * 90
        for x in f:
            if x < 1260:
                pi, sq = divmod(x, 90)
                board[sq] = pi + 1 if pi < 7 else -(pi - 7 + 1)
                bf[sq] = x
        threats = [int(t) for t in az_threat_features(board, 0)]
        mi = [int(m) for m in samples.move_indices[samples.move_offsets[i]:samples.move_offsets[i + 1]]]
        pt = [F32(p) for p in samples.policy[samples.move_offsets[i]:samples.move_offsets[i + 1]]]
        per.append((i, f, board, bf, threats, mi, pt))
    B = len(rows)
    Fm = max([len(p[1]) for p in per] + [1])
    Mm = max([sum(m < 2086 for m in p[5]) for p in per] + [1])
    Tm = max([len(p[4]) for p in per] + [1])
    out = dict(
        feature_items=np.full((B, Fm), PAD, np.uint32), value_threat_indices=np.full((B, Tm), PAD, np.uint32),
        policy_items=np.zeros((B, Mm), np.int64), policy_sparse_indices=np.full((B, Mm, 7), SPARSE_TABLE - 1, np.int64),
        policy_tactical_indices=np.full((B, Mm, 2), TACTICAL, np.int64), policy_targets=np.zeros((B, Mm), F32),
        policy_mask=np.full((B, Mm), F32(-1.0e9), F32), value_wdl=np.zeros((B, 3), F32), values=np.zeros(B, F32),
        rule_context=np.zeros((B, 7), F32), policy_weights=np.ones(B, F32), value_weights=np.ones(B, F32),
        value_phase_masks=np.zeros((B, 3), F32))
    for row, (i, f, board, bf, threats, mi, pt) in enumerate(per):
        us = them = 4
        for x in f:
            if x < 1260:
                pi, sq = divmod(x, 90)
                if pi == 0:
                    us = _general_bucket(0, sq)
                if pi == 7:
                    them = _general_bucket(7, sq)
        for k, x in enumerate(f):
            if x < 1260:
                out["feature_items"][row, k] = x | us << 11 | them << 15
        out["value_threat_indices"][row, :len(threats)] = threats
        off = 0
        for m, target in zip(mi, pt):
            if m >= 2086:
                continue
            out["policy_targets"][row, off] = _max0(target)
            out["policy_mask"][row, off] = 0.0
            frm, to = divmod(int(moves_map[m]), 90)
            mf = bf[frm]
            valid = mf >= 0 and mf // 90 < 7
            cf = ct = cc = 0
            cap = False
            if valid:
                cf, ct = mf, (mf // 90) * 90 + to
                if bf[to] >= 0:
                    cc, cap = bf[to], True
            out["policy_items"][row, off] = (m | cf << 12 | ct << 23 | cc << 34 | int(valid) << 45
                                             | int(cap) << 46 | 1 << 47)
            if valid:
                piece = mf // 90
                pair = us * 9 + them
                king = 89 - ((7 + them // 3) * 9 + 3 + them % 3)
                before = abs(frm // 9 - king // 9) + abs(frm % 9 - king % 9)
                after = abs(to // 9 - king // 9) + abs(to % 9 - king % 9)
                approach = min(max(before - after, -2), 2) + 2
                distance = min(after, 5)
                mp, mk = 2086 * 14, 2086 * 81
                doff = mp + mk + 14 * 81
                out["policy_sparse_indices"][row, off] = [
                    ((m * 14 + piece) * 9 + us) * 9 + them,
                    SPARSE_MAIN + m * 15 + (cc // 90 if cap else 14),
                    SPARSE_TABLE + m * 14 + piece,
                    SPARSE_TABLE + mp + m * 81 + pair,
                    SPARSE_TABLE + mp + mk + piece * 81 + pair,
                    SPARSE_TABLE + doff + piece * 6 + distance,
                    SPARSE_TABLE + doff + 14 * 6 + piece * 5 + approach]
                info = az_policy_moves(board, 0, np.array([[frm, to]], np.uint8))[0, 0]
                sig = int(info >> 20) & 0x3F
                out["policy_tactical_indices"][row, off] = [(m * 7 + piece) * 64 + sig, TACTICAL_EXACT + piece * 64 + sig]
            off += 1
        if off:
            t = out["policy_targets"][row]
            s = F32(0.0)
            for k in range(off):
                s = F32(s + t[k])
            if np.isfinite(s) and s > F32(1e-12):
                for k in range(off):
                    t[k] = _max0(F32(t[k] / s))
            else:
                t[:off] = F32(1.0) / F32(off)
        w = [_max0(x) for x in samples.value_wdl[i]]
        ws = F32(F32(w[0] + w[1]) + w[2])
        out["value_wdl"][row] = [F32(x / ws) for x in w] if np.isfinite(ws) and ws > F32(1e-6) else [0, 1, 0]
        out["values"][row] = min(max(F32(samples.value[i]), F32(-1.0)), F32(1.0))
        out["rule_context"][row] = samples.rule_context[i]
        out["policy_weights"][row] = _max0(samples.policy_weight[i])
        out["value_weights"][row] = _max0(samples.value_weight[i])
        ply = int(samples.ply[i])
        out["value_phase_masks"][row, 0 if ply < 40 else (1 if ply < 120 else 2)] = 1.0
    return out
