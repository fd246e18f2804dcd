"""The AdamW restatement (oracle.adamw, candle-nn's AdamW::step operation
order) pinned against torch.optim.AdamW in float64: same published
algorithm (decoupled weight decay, bias-corrected moments)."""
import numpy as np
import torch

import oracle


def test_adamw_matches_torch_float64_over_steps():
    rng = np.random.default_rng(5)
    p0 = rng.standard_normal(1000).astype(np.float32)
    p, m, v = p0.copy(), np.zeros_like(p0), np.zeros_like(p0)
    tp = torch.tensor(p0, dtype=torch.float64, requires_grad=True)
    opt = torch.optim.AdamW([tp], lr=3e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    for step in range(1, 6):
        g = rng.standard_normal(1000).astype(np.float32) * 0.1
        g[:7] = 0.0
        oracle.adamw(p, m, v, g, 3e-3, step=step)
        tp.grad = torch.tensor(g, dtype=torch.float64)
        opt.step()
        np.testing.assert_allclose(p, tp.detach().numpy(), rtol=2e-6, atol=2e-7)
