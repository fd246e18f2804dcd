"""Independent numpy restatement of the quantised and fp32 HalfKA networks,
used to cross-check the C oracle (vectorised, different code path)."""
import numpy as np


def _list_ids(offsets):
    counts = np.diff(offsets.astype(np.int64))
    return np.repeat(np.arange(len(counts)), counts), counts


def q_forward(w, pos):
    n = pos.n
    ids, counts = _list_ids(pos.offsets)
    sums = np.zeros((2 * n, 1024), np.int64)
    np.add.at(sums, ids, w.ft_weight[pos.indices.astype(np.int64)].astype(np.int64))
    acc = sums + w.ft_bias.astype(np.int64)
    acc = ((acc + 32768) % 65536) - 32768
    acc = acc.reshape(n, 2, 1024)
    a = np.clip(acc[:, :, :512], 0, 127)
    b = np.clip(acc[:, :, 512:], 0, 127)
    x = ((a * b) >> 7).reshape(n, 1024)
    n0 = counts.reshape(n, 2)[:, 0]
    bucket = np.minimum((np.maximum(n0, 1) - 1) >> 1, 15)
    y1 = np.einsum("nki,ni->nk", w.l1_weight[bucket].astype(np.int64), x) + w.l1_bias[bucket]
    y1 = np.clip(y1 >> 6, 0, 127)
    y2 = np.einsum("nmk,nk->nm", w.l2_weight[bucket].astype(np.int64), y1) + w.l2_bias[bucket]
    y2 = np.clip(y2 >> 6, 0, 127)
    out = np.einsum("nm,nm->n", w.l3_weight[bucket].astype(np.int64), y2) + w.l3_bias[bucket]
    return out.astype(np.int32), acc.astype(np.int16)


def q_update(w, batch):
    n = batch.n
    par = batch.parent.reshape(2 * n, 1024).astype(np.int64)
    refresh = (batch.flags & 1).astype(bool)
    base = np.where(refresh[:, None], w.ft_bias.astype(np.int64)[None, :], par)
    rid, _ = _list_ids(batch.rem_offsets)
    aid, _ = _list_ids(batch.add_offsets)
    keep = ~refresh[rid]
    np.subtract.at(base, rid[keep], w.ft_weight[batch.rem.astype(np.int64)[keep]].astype(np.int64))
    np.add.at(base, aid, w.ft_weight[batch.add.astype(np.int64)].astype(np.int64))
    acc = (((base + 32768) % 65536) - 32768).reshape(n, 2, 1024)
    a = np.clip(acc[:, :, :512], 0, 127)
    b = np.clip(acc[:, :, 512:], 0, 127)
    x = ((a * b) >> 7).reshape(n, 1024)
    bucket = np.minimum((np.maximum(batch.count0.astype(np.int64), 1) - 1) >> 1, 15)
    y1 = np.clip((np.einsum("nki,ni->nk", w.l1_weight[bucket].astype(np.int64), x) + w.l1_bias[bucket]) >> 6, 0, 127)
    y2 = np.clip((np.einsum("nmk,nk->nm", w.l2_weight[bucket].astype(np.int64), y1) + w.l2_bias[bucket]) >> 6, 0, 127)
    out = np.einsum("nm,nm->n", w.l3_weight[bucket].astype(np.int64), y2) + w.l3_bias[bucket]
    return acc.astype(np.int16), out.astype(np.int32)


def f_forward(w, pos):
    """float64 evaluation of the fp32 network (a tolerance reference)."""
    n = pos.n
    ids, counts = _list_ids(pos.offsets)
    sums = np.zeros((2 * n, 256), np.float64)
    np.add.at(sums, ids, w.ft_weight[pos.indices.astype(np.int64)].astype(np.float64))
    acc = (sums + w.ft_bias).reshape(n, 2, 256)
    x = np.clip(acc, 0, 1).reshape(n, 512)
    n0 = counts.reshape(n, 2)[:, 0]
    bucket = np.minimum((np.maximum(n0, 1) - 1) >> 2, 7)
    h1 = np.clip(np.einsum("nki,ni->nk", w.l1_weight[bucket].astype(np.float64), x) + w.l1_bias[bucket], 0, 1)
    h2 = np.clip(np.einsum("nmk,nk->nm", w.l2_weight[bucket].astype(np.float64), h1) + w.l2_bias[bucket], 0, 1)
    return np.einsum("nm,nm->n", w.l3_weight[bucket].astype(np.float64), h2) + w.l3_bias[bucket]


def pool_item_rows(packed):
    feature = packed & 0x7FF
    us = (packed >> 11) & 0xF
    them = (packed >> 15) & 0xF
    piece, square = feature // 90, feature % 90
    return [feature, 1260 + piece, 1274 + square // 9, 1284 + square % 9, 1293 + us * 14 + piece,
            1293 + (9 + them) * 14 + piece]


def feature_pool_fwd(tables, items):
    """Sequential float32 restatement of FeaturePool::cpu_fwd
    (src/az/fused_feature_pool.rs:169-198)."""
    batch, ic = items.shape
    hidden = tables.shape[1]
    out = np.zeros((batch, hidden), np.float32)
    for b in range(batch):
        for i in range(ic):
            p = int(items[b, i])
            if p == 0xFFFFFFFF:
                continue
            rows = pool_item_rows(p)
            for h in range(hidden):
                o = out[b, h]
                for r in rows:
                    o = np.float32(o + tables[r, h])
                out[b, h] = o
    return out


def feature_pool_bwd(items, grad_out, n_rows=1545):
    """Sequential float32 restatement of FeaturePoolGrad::cpu_fwd
    (src/az/fused_feature_pool.rs:231-260)."""
    batch, ic = items.shape
    hidden = grad_out.shape[1]
    g = np.zeros((n_rows, hidden), np.float32)
    for b in range(batch):
        for i in range(ic):
            p = int(items[b, i])
            if p == 0xFFFFFFFF:
                continue
            for r in pool_item_rows(p):
                g[r] = g[r] + grad_out[b]
    return g
