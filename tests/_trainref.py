"""Batches for the training-step parity tests.

The network is piecewise linear: a hidden unit whose pre-activation lies
within rounding distance of a clamp boundary (0 or 1) can take a different
mask in two correct implementations that sum in different orders, and its
whole position's gradient then differs.  `safe_batch` drops such positions
(pre-activation within `margin` of a boundary, computed in fp64 from the exact
fp32/bf16 activations both implementations share) so the comparison tests the
arithmetic, not the knife edge.
"""
import numpy as np

import oracle
from chineseai_b200 import synth, train


def select(pos, keep):
    idx, off = [], [0]
    for b in np.flatnonzero(keep):
        for s in range(2):
            seg = pos.indices[pos.offsets[2 * b + s]: pos.offsets[2 * b + s + 1]]
            idx.append(seg)
            off.append(off[-1] + len(seg))
    idx = np.concatenate(idx) if idx else np.zeros(0, np.uint16)
    return synth.Positions(idx.astype(np.uint16), np.array(off, np.uint32))


def activations(params, pos):
    p = train.split(params)
    ftb = oracle.bf16_round(p["ft"])
    bb = oracle.bf16_round(p["ft_bias"])
    n = pos.n
    counts = np.diff(pos.offsets.astype(np.int64))
    acc = np.broadcast_to(bb, (2 * n, 1024)).astype(np.float32).copy()
    for k in range(int(counts.max()) if len(counts) else 0):
        lists = np.flatnonzero(counts > k)
        rows = pos.indices[pos.offsets[lists].astype(np.int64) + k]
        acc[lists] = acc[lists] + ftb[rows]
    return oracle.bf16_round(acc).reshape(n, 2, 1024)


def knife_edge(params, pos, margin=1e-5):
    p = train.split(params)
    a = activations(params, pos)
    u = np.clip(a, 0, 1)
    x = oracle.bf16_round((u[:, :, :512] * u[:, :, 512:]).reshape(pos.n, 1024)).astype(np.float64)
    n0 = np.diff(pos.offsets.astype(np.int64)).reshape(pos.n, 2)[:, 0]
    bk = np.minimum((np.maximum(n0, 1) - 1) >> 1, 15)
    z1 = np.empty((pos.n, 16))
    z2 = np.empty((pos.n, 32))
    for b in np.unique(bk):
        sel = bk == b
        z1[sel] = x[sel] @ p["w1"][b].astype(np.float64).T + p["b1"][b]
        z2[sel] = np.clip(z1[sel], 0, 1) @ p["w2"][b].astype(np.float64).T + p["b2"][b]
    near = lambda z: (np.abs(z) < margin) | (np.abs(z - 1) < margin)
    return near(z1).any(1) | near(z2).any(1)


def safe_batch(params, n, seed, margin=1e-5):
    pos = synth.positions(n, seed)
    t = train.targets(n, seed + 100)
    bad = knife_edge(params, pos, margin)
    return select(pos, ~bad), t[~bad], int(bad.sum())
