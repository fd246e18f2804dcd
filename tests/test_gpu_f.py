"""GPU parity of the fp32 evaluator against the oracle (tolerance 1e-4
relative, 1e-6 absolute: the stack's dot products sum in a different order)."""
import os

import numpy as np
import pytest

import oracle
from chineseai_b200 import synth
from chineseai_b200.fp32 import FloatNnue

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
RTOL, ATOL = 1e-4, 1e-6


@pytest.fixture(scope="module")
def fmodel(fweights):
    m = FloatNnue(fweights, 0)
    yield m
    m.close()


def test_golden(fmodel):
    g = np.load(GOLDEN)
    out = fmodel.forward_positions(synth.Positions(g["q_idx"], g["q_off"]))
    np.testing.assert_allclose(out, g["f_out"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("n,seed", [(1, 2), (100, 3), (4096, 1), (140_000, 5)])
def test_random(fmodel, fweights, n, seed):
    pos = synth.positions(n, seed)
    out = fmodel.forward_positions(pos)
    st, ref, _ = oracle.f_forward(fweights, pos)
    assert st == 0
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)


def test_all_buckets(fmodel, fweights):
    rng = np.random.default_rng(3)
    idx, off = [], [0]
    for n0 in range(0, 36):
        for s in range(2):
            k = n0 if s == 0 else 17
            idx += list(np.sort(rng.choice(11340, size=k, replace=False)))
            off.append(len(idx))
    pos = synth.Positions(np.array(idx, np.uint16), np.array(off, np.uint32))
    out = fmodel.forward_positions(pos)
    st, ref, _ = oracle.f_forward(fweights, pos)
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)


def test_bad_offsets_and_indices_are_reported(fmodel):
    from chineseai_b200._lib import CnnueError
    idx = np.array([5, 7, 11339, 3], np.uint16)
    with pytest.raises(CnnueError):  # a list that ends before it starts
        fmodel.forward_positions(synth.Positions(idx, np.array([0, 3, 2, 4], np.uint32)[:3].copy()))
    with pytest.raises(CnnueError):  # a feature past 11340
        fmodel.forward_positions(synth.Positions(np.array([5, 11340], np.uint16), np.array([0, 1, 2], np.uint32)))
