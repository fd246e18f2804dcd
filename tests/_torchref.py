"""torch autograd restatement of the training step's loss (CPU), used to check
the oracle's hand-written backward.  The FT activations are computed in fp32
in the oracle's order so their bf16 rounding matches; the stack runs in fp64;
bf16 roundings pass gradients straight through; clamp masks are strict."""
import numpy as np
import torch

import oracle
from chineseai_b200.train import COLS, LAYOUT, N_FEATURES


def _ste_clamp(v):
    inside = (v > 0) & (v < 1)
    return torch.where(inside, v, v.detach().clamp(0.0, 1.0))


def loss_and_grad(params: np.ndarray, pos, target: np.ndarray):
    n = pos.n
    ft32 = params[: N_FEATURES * COLS].reshape(N_FEATURES, COLS)
    bias32 = params[N_FEATURES * COLS: N_FEATURES * COLS + COLS]
    ft_b = oracle.bf16_round(ft32)
    bias_b = oracle.bf16_round(bias32)
    # fp32 activations in the oracle's order
    a_val = np.zeros((n, 2, COLS), np.float32)
    for b in range(n):
        for p in range(2):
            acc = bias_b.copy()
            for i in range(pos.offsets[2 * b + p], pos.offsets[2 * b + p + 1]):
                acc = acc + ft_b[pos.indices[i]]
            a_val[b, p] = oracle.bf16_round(acc)
    W = torch.tensor(params, dtype=torch.float64, requires_grad=True)
    views, o = {}, 0
    for name, shape in LAYOUT:
        k = int(np.prod(shape))
        views[name] = W[o:o + k].view(*shape)
        o += k
    lin = []
    for b in range(n):
        row = []
        for p in range(2):
            s = views["ft_bias"]
            for i in range(pos.offsets[2 * b + p], pos.offsets[2 * b + p + 1]):
                s = s + views["ft"][int(pos.indices[i])]
            row.append(s)
        lin.append(torch.stack(row))
    lin = torch.stack(lin)  # (n, 2, 1024)
    a = torch.tensor(a_val, dtype=torch.float64) + lin - lin.detach()
    u = _ste_clamp(a)
    x = (u[:, :, :512] * u[:, :, 512:]).reshape(n, 1024)
    x = x + (torch.tensor(oracle.bf16_round(x.detach().numpy().astype(np.float32)), dtype=torch.float64) - x.detach())
    n0 = np.diff(pos.offsets.astype(np.int64)).reshape(n, 2)[:, 0]
    bk = torch.tensor(np.minimum((np.maximum(n0, 1) - 1) >> 1, 15))
    z1 = torch.einsum("nki,ni->nk", views["w1"][bk], x) + views["b1"][bk]
    h1 = _ste_clamp(z1)
    z2 = torch.einsum("nmk,nk->nm", views["w2"][bk], h1) + views["b2"][bk]
    h2 = _ste_clamp(z2)
    s = (views["w3"][bk] * h2).sum(1) + views["b3"][bk]
    sg = torch.sigmoid(s / 400.0)
    loss = ((sg - torch.tensor(target, dtype=torch.float64)) ** 2).mean()
    loss.backward()
    return float(loss.detach()), W.grad.numpy()
