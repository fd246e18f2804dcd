"""GPU parity of the tcgen05 ResNet (policy/value inference) against the oracle.

The oracle accumulates in fp32 from the same bf16 weights and rounds every
trunk activation to bf16 as the device stores it, so the two differ only by
the tensor cores' summation order (and the rare bf16 rounding flips that
follow from it).  Tolerances: logits within 1e-2 of the largest logit
magnitude (relative), policy probabilities within 1e-3, values within 5e-3.
Batches cover partial 128-square tiles (B = 1, 3, 37) and the empty board."""
import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import resnet

pytestmark = pytest.mark.gpu

_M = {}


def _model():
    if "m" not in _M:
        w = resnet.ResNetWeights.synthetic(5)
        _M["m"] = (w, resnet.ResNetModel(w, device=0))
    return _M["m"]


@pytest.mark.parametrize("batch,seed", [(1, 6), (3, 7), (37, 8), (64, 9)])
def test_resnet_matches_oracle(batch, seed):
    w, model = _model()
    planes = resnet.synthetic_planes(batch, seed)
    if batch >= 3:
        planes[1] = 0  # an empty board, Red to move
    dev = torch.from_numpy(planes.view(np.int16)).cuda()
    probs, logits, value = model.forward(dev, with_logits=True)
    assert model.read_status() == 0
    lg, pr, vpre, v, _ = oracle.rn_forward(w, planes)
    g_logits = logits.cpu().numpy()
    scale = max(1.0, float(np.abs(lg).max()))
    assert np.abs(g_logits - lg).max() <= 1e-2 * scale
    np.testing.assert_allclose(probs.cpu().numpy(), pr, atol=1e-3, rtol=0)
    np.testing.assert_allclose(value.cpu().numpy(), v, atol=5e-3, rtol=0)
    np.testing.assert_allclose(probs.sum(1).cpu().numpy(), 1.0, atol=1e-4)


def test_resnet_is_deterministic_and_batch_independent():
    w, model = _model()
    planes = resnet.synthetic_planes(40, 11)
    dev = torch.from_numpy(planes.view(np.int16)).cuda()
    p1, l1, v1 = model.forward(dev, with_logits=True)
    p2, l2, v2 = model.forward(dev, with_logits=True)
    assert torch.equal(l1, l2) and torch.equal(v1, v2)
    # a board's result does not depend on its neighbours in the batch
    p3, l3, v3 = model.forward(dev[5:6].contiguous(), with_logits=True)
    assert torch.equal(l3[0], l1[5]) and torch.equal(v3[0], v1[5])
