"""chineseai_b200: B200-native (sm_100a) NNUE evaluation hot path of mycve/chineseai.

The compute lives in libcnnue.so (CUDA kernels behind the C ABI of
include/cnnue.h); this package is the Python host side over that ABI.
"""
from ._lib import CnnueError, LIB_PATH, lib  # noqa: F401

__version__ = "0.1.0"
