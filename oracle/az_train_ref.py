"""AZ-NNUE training step restated in plain torch on the CPU - TEST
INFRASTRUCTURE ONLY.

AzCandleModel::forward (src/az/candle_model.rs:46-147) with its custom ops
written as gathers: feature_pool's six rows per item (fused_feature_pool.rs:
389-403), sparse_pool, fused_policy's three terms (fused_policy.rs:178-241),
sparse / tactical lookups; then compute_batch_loss
(src/az/train_gpu_candle.rs:221-305).  Gradients come from torch autograd of
this forward, independent of the CUDA backward kernels; the AdamW update is
the oracle's C restatement (oracle.adamw).  Runs in float64 by default.
"""
from __future__ import annotations

import numpy as np
import torch

PAD = 0xFFFFFFFF


def _pool_rows(items: np.ndarray):
    """feature_pool item -> its six rows of the [1545, H] table; mask of real items."""
    it = items.astype(np.int64)
    valid = it != PAD
    f = it & 0x7FF
    us = (it >> 11) & 0xF
    them = (it >> 15) & 0xF
    piece, sq = f // 90, f % 90
    rows = np.stack([f, 1260 + piece, 1274 + sq // 9, 1284 + sq % 9, 1293 + us * 14 + piece,
                     1293 + (9 + them) * 14 + piece], -1)
    rows[~valid] = 0
    return torch.from_numpy(rows), torch.from_numpy(valid)


def forward(t, b, dtype=torch.float64):
    """t: the 22 tensors (torch, requires_grad as wanted); b: PackedBatch.
    Returns (value_logits [B, 3], policy_logits [B, M])."""
    h = t[0].shape[1]
    ft = torch.cat([t[0], t[1], t[2], t[3], t[4]], 0)
    rows, valid = _pool_rows(b.feature_items)
    board_pre = (ft[rows] * valid[..., None, None].to(dtype)).sum((1, 2)) + t[6]
    acc_ctx = board_pre @ t[17].t()
    rule = torch.from_numpy(b.rule_context).to(dtype)
    sparse_hidden = torch.relu(board_pre + rule @ t[5])
    rms = torch.sqrt((sparse_hidden * sparse_hidden).mean(1, keepdim=True) + 1e-6)
    hidden = sparse_hidden / rms
    value_head = torch.relu(hidden @ t[7].t() + t[8])
    value_logits = value_head @ t[9].t()
    ti = b.value_threat_indices.astype(np.int64)
    tv = torch.from_numpy(ti != PAD)
    ti[ti == PAD] = 0
    threat_acc = (t[10][torch.from_numpy(ti)] * tv[..., None].to(dtype)).sum(1)
    act = threat_acc.clamp(0.0, 1.0)
    pair = torch.cat([act, act * act], 1)
    value_logits = value_logits + pair @ t[11].t()
    cs = min(32, h)
    psp = t[0][:, :cs]
    if cs < 32:
        psp = torch.cat([psp, psp.new_zeros(1260, 32 - cs)], 1)
    ctx = torch.cat([hidden @ t[15].t() + pair @ t[12].t(), acc_ctx], 1)
    acc_feature = t[0] @ t[17].t()
    items = b.policy_items.astype(np.uint64)
    pv = torch.from_numpy(((items >> np.uint64(47)) & np.uint64(1)).astype(bool))
    mvv = torch.from_numpy(((items >> np.uint64(45)) & np.uint64(1)).astype(np.float64)).to(dtype)
    cpv = torch.from_numpy(((items >> np.uint64(46)) & np.uint64(1)).astype(np.float64)).to(dtype)
    mv = torch.from_numpy((items & np.uint64(0xFFF)).astype(np.int64))
    fr = torch.from_numpy(((items >> np.uint64(12)) & np.uint64(0x7FF)).astype(np.int64))
    to = torch.from_numpy(((items >> np.uint64(23)) & np.uint64(0x7FF)).astype(np.int64))
    cp = torch.from_numpy(((items >> np.uint64(34)) & np.uint64(0x7FF)).astype(np.int64))
    delta = psp[to] - psp[fr] - cpv[..., None] * psp[cp]
    logit = t[13][mv] + mvv * (
        (delta * t[14]).sum(-1)
        + (ctx[:, None, :16] * t[16][mv]).sum(-1)
        + ((ctx[:, None, 16:] + acc_feature[to] - acc_feature[fr] - cpv[..., None] * acc_feature[cp])
           * t[18][mv]).sum(-1))
    policy_logits = torch.where(pv, logit, torch.zeros_like(logit))
    sparse = torch.cat([t[19], t[20]])
    policy_logits = policy_logits + sparse[torch.from_numpy(b.policy_sparse_indices)].sum(-1)
    tactical = torch.cat([t[21], t[21].new_zeros(1)])
    policy_logits = policy_logits + tactical[torch.from_numpy(b.policy_tactical_indices)].sum(-1)
    return value_logits, policy_logits


def loss(t, b, value_weight=1.0, policy_weight=1.0, dtype=torch.float64):
    value_logits, policy_logits = forward(t, b, dtype)
    T = lambda a: torch.from_numpy(np.asarray(a)).to(dtype)  # noqa: E731
    vlp = torch.log_softmax(value_logits, 1)
    value_ce = -(T(b.value_wdl) * vlp).sum(1)
    lp = torch.log_softmax(policy_logits + T(b.policy_mask), 1)
    policy_ce = -(T(b.policy_targets) * lp).sum(1)
    total = (value_ce * T(b.value_weights)).sum() * max(value_weight, 0.0) + \
        (policy_ce * T(b.policy_weights)).sum() * max(policy_weight, 0.0)
    return total / b.batch_size, value_logits, policy_logits


def gradients(tensors, b, value_weight=1.0, policy_weight=1.0, dtype=torch.float64):
    """(loss, [22 gradient arrays]) of the restated step."""
    t = [torch.tensor(np.asarray(x), dtype=dtype, requires_grad=True) for x in tensors]
    lv, _, _ = loss(t, b, value_weight, policy_weight, dtype)
    lv.backward()
    return float(lv.detach()), [x.grad.numpy() for x in t]
