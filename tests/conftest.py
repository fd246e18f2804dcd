import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def qweights():
    from chineseai_b200 import synth
    return synth.quantized_weights(2)


@pytest.fixture(scope="session")
def fweights():
    from chineseai_b200 import synth
    return synth.float_weights(2)


@pytest.fixture(scope="session")
def qmodel(qweights):
    from chineseai_b200.quantized import QuantizedNnue
    m = QuantizedNnue(qweights, device=0)
    yield m
    m.close()
