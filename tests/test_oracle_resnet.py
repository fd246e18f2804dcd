"""CPU checks of the ResNet oracle: an independent numpy restatement (im2col
matmuls in float64, the same bf16 rounding of every trunk activation) agrees
with it within the tolerance the GPU test uses, which also measures how far
two correct summation orders drift apart through 21 bf16-rounded layers; the
synthetic generators are deterministic and bf16-valued."""
import numpy as np

import oracle
from chineseai_b200 import resnet


def _bf16(x):
    u = np.asarray(x, np.float32).copy().view(np.uint32)
    u += np.uint32(0x7FFF) + ((u >> 16) & 1)
    u &= np.uint32(0xFFFF0000)
    return u.view(np.float32)


def _im2col(x, cin):
    xp = np.zeros((cin, 12, 11), x.dtype)
    xp[:, 1:11, 1:10] = x.reshape(cin, 10, 9)
    cols = np.zeros((90, cin, 3, 3), x.dtype)
    for kh in range(3):
        for kw in range(3):
            cols[:, :, kh, kw] = xp[:, kh:kh + 10, kw:kw + 9].reshape(cin, 90).T
    return cols.reshape(90, cin * 9)


def _numpy_net(w, planes):
    x = resnet.bf16_to_float(planes).reshape(15, 90).astype(np.float64)

    def conv(x, cin, W, b, res=None):
        y = _im2col(x, cin) @ W.reshape(128, cin * 9).astype(np.float64).T + b
        if res is not None:
            y = y + res.T
        return _bf16(np.maximum(y, 0)).astype(np.float64).T

    x = conv(x, 15, w.stem_w, w.stem_b)
    for blk in range(10):
        h = conv(x, 128, w.block_w[blk, 0], w.block_b[blk, 0])
        x = conv(h, 128, w.block_w[blk, 1], w.block_b[blk, 1], x)
    pc = np.maximum(w.policy_conv_w.astype(np.float64) @ x + w.policy_conv_b[:, None], 0).reshape(-1)
    logits = w.policy_fc_w.astype(np.float64) @ pc + w.policy_fc_b
    vc = np.maximum(w.value_conv_w.astype(np.float64) @ x + w.value_conv_b[0], 0)
    hid = np.maximum(w.value_fc1_w.astype(np.float64) @ vc + w.value_fc1_b, 0)
    return logits, np.tanh(w.value_fc2_w @ hid + w.value_fc2_b[0])


def test_oracle_matches_independent_numpy_restatement():
    w = resnet.ResNetWeights.synthetic(5)
    planes = resnet.synthetic_planes(4, 10)
    planes[2] = 0
    lg, pr, vpre, v, _ = oracle.rn_forward(w, planes)
    scale = max(1.0, float(np.abs(lg).max()))
    for i in range(4):
        ref_lg, ref_v = _numpy_net(w, planes[i])
        assert np.abs(ref_lg - lg[i]).max() <= 1e-2 * scale
        assert abs(ref_v - v[i]) <= 5e-3
        e = np.exp(lg[i] - lg[i].max())
        np.testing.assert_allclose(pr[i], e / e.sum(), atol=1e-6)


def test_generators_are_deterministic_and_bf16_valued():
    a, b = resnet.ResNetWeights.synthetic(5), resnet.ResNetWeights.synthetic(5)
    for x, y in zip(a.arrays(), b.arrays()):
        np.testing.assert_array_equal(x, y)
        assert not (x.view(np.uint32) & 0xFFFF).any()
    p = resnet.synthetic_planes(200, 6)
    np.testing.assert_array_equal(p, resnet.synthetic_planes(200, 6))
    f = resnet.bf16_to_float(p)
    assert set(np.unique(f)) <= {0.0, 1.0}
    pieces = f[:, :14].sum(axis=(1, 2, 3))
    assert pieces.max() <= 32 and pieces.min() >= 0
    assert (f[:, :14].sum(axis=1) <= 1).all()  # one piece per square
    stm = f[:, 14].reshape(200, -1)
    assert ((stm == 0).all(1) | (stm == 1).all(1)).all()
