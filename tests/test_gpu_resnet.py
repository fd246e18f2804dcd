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


def test_resnet_back_to_back_forwards_identical():
    # forwards of two alternating batches queued with no host synchronisation:
    # every kernel of a forward (the head kernels are programmatic dependents)
    # must read its predecessor's finished output, so each result equals the
    # synchronised first result of its batch bit for bit
    w, model = _model()
    a = torch.from_numpy(resnet.synthetic_planes(1024, 21).view(np.int16)).cuda()
    b = torch.from_numpy(resnet.synthetic_planes(1024, 22).view(np.int16)).cuda()
    ref = []
    for x in (a, b):
        out = model.forward(x, with_logits=True)
        torch.cuda.synchronize()
        ref.append([t.clone() for t in out])
    outs = [model.forward(a if i % 2 == 0 else b, with_logits=True) for i in range(16)]
    torch.cuda.synchronize()
    for i, out in enumerate(outs):
        for got, want in zip(out, ref[i % 2]):
            assert torch.equal(got, want), i


def _check_against_oracle(w, planes, probs, logits, value):
    lg, pr, _, v, _ = oracle.rn_forward(w, planes)
    scale = max(1.0, float(np.abs(lg).max()))
    assert np.abs(logits - lg).max() <= 1e-2 * scale
    np.testing.assert_allclose(probs, pr, atol=1e-3, rtol=0)
    np.testing.assert_allclose(value, v, atol=5e-3, rtol=0)


@pytest.mark.parametrize("kind", ["tile", "persistent"])
def test_square_major_conv_kernels_match_oracle(kind):
    """The two square-major conv kernels (one TMA box per tap, edge rows
    zeroed in shared memory) against the oracle."""
    w, model = _model()
    planes = resnet.synthetic_planes(37, 13)
    dev = torch.from_numpy(planes.view(np.int16)).cuda()
    model.set_conv_kernel(kind)
    try:
        probs, logits, value = model.forward(dev, with_logits=True)
        assert model.read_status() == 0
    finally:
        model.set_conv_kernel("halo")
    _check_against_oracle(w, planes, probs.cpu().numpy(), logits.cpu().numpy(), value.cpu().numpy())


def test_halo_kernel_many_pairs_per_cta():
    """700 boards: 88 groups of 8 (the last one partial), 77,440 padded rows,
    303 row pairs, so every CTA of the persistent halo kernel runs two or
    three pairs and both halo buffers and TMEM accumulators turn over.  A
    sample of boards is checked against the oracle (boards are independent),
    and each board equals its result in a batch of one."""
    w, model = _model()
    planes = resnet.synthetic_planes(700, 14)
    planes[699] = 0
    dev = torch.from_numpy(planes.view(np.int16)).cuda()
    probs, logits, value = model.forward(dev, with_logits=True)
    assert model.read_status() == 0
    sample = np.array([0, 1, 7, 8, 255, 256, 351, 352, 517, 694, 695, 696, 699])
    _check_against_oracle(w, planes[sample], probs.cpu().numpy()[sample], logits.cpu().numpy()[sample],
                          value.cpu().numpy()[sample])
    for b in (0, 352, 699):
        p1, l1, v1 = model.forward(dev[b:b + 1].contiguous(), with_logits=True)
        assert torch.equal(l1[0], logits[b]) and torch.equal(v1[0], value[b])


def test_resnet_full_config_batch_1024_every_board():
    """The configured leaf batch, 1024 boards (128 whole 8-board groups),
    compared board by board with the oracle at the tolerances above; the
    batch includes an empty board at both ends of the buffer."""
    w, model = _model()
    planes = resnet.synthetic_planes(1024, 21)
    planes[0] = 0
    planes[-1] = 0
    dev = torch.from_numpy(planes.view(np.int16)).cuda()
    probs, logits, value = model.forward(dev, with_logits=True)
    assert model.read_status() == 0
    lg, pr, _, v, _ = oracle.rn_forward(w, planes)
    g_logits, g_probs, g_value = logits.cpu().numpy(), probs.cpu().numpy(), value.cpu().numpy()
    scale = np.maximum(1.0, np.abs(lg).max(axis=1))
    per_board = np.abs(g_logits - lg).max(axis=1) / scale
    assert per_board.max() <= 1e-2, (int(per_board.argmax()), float(per_board.max()))
    np.testing.assert_allclose(g_probs, pr, atol=1e-3, rtol=0)
    np.testing.assert_allclose(g_value, v, atol=5e-3, rtol=0)
