"""CPU tests of the C ABI boundary: the library loads, exports every symbol
the headers declare, validates arguments without a GPU, and its workload
generators are deterministic."""
import ctypes as C
import glob
import os
import re

import numpy as np

from chineseai_b200 import _lib, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(cnnue_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each
    assert names <= set(_lib.SIGNATURES), sorted(names - set(_lib.SIGNATURES))


def test_status_strings_and_version():
    assert _lib.status_string(0) == "ok"
    assert "index" in _lib.status_string(2)
    assert _lib.lib().cnnue_version().decode() == "0.1.0"


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _lib.lib()
    h = C.c_void_p()
    assert lib.cnnue_q_model_create(None, 0, C.byref(h)) == 1
    assert lib.cnnue_f_model_create(None, 0, C.byref(h)) == 1
    assert lib.cnnue_q_forward(None, None, 0, None, 10, None, None, 0, None) == 1
    assert lib.cnnue_q_forward_host(None, None, 0, None, 1, None, None) == 1
    assert lib.cnnue_q_ctx_create(None, 10, 10, C.byref(h)) == 1
    assert lib.cnnue_q_forward_host_async(None, None, 0, None, 1, None, None) == 1
    st = C.c_int(0)
    assert lib.cnnue_q_ctx_wait(None, 0, C.byref(st)) == 1
    assert lib.cnnue_feature_pool_fwd(None, None, -1, 1, 1, None, None, None) == 1
    assert lib.cnnue_read_status(None, None, None) == 1
    assert lib.cnnue_sparse_pool_bwd(None, None, 20000, 1, 1, 1, None, None, 0, None) == 1
    assert "null" in _lib.last_error() or "rows" in _lib.last_error()


def test_workspace_sizes():
    lib = _lib.lib()
    a = lib.cnnue_q_workspace_bytes(1)
    b = lib.cnnue_q_workspace_bytes(65536)
    assert 512 < a < b
    assert b >= 65536 * 6
    assert lib.cnnue_feature_pool_bwd_workspace_bytes(1024, 32, 128) > 1024 * 32 * 6 * 4
    # fp32 forward: the 512-byte header, the clipped FT outputs [n][512] fp32
    # and the bucket lists [8][n] u32
    for n in (1, 4096, 140_000):
        assert lib.cnnue_f_workspace_bytes(n) >= 512 + n * 512 * 4 + 8 * n * 4


def test_splitmix64_matches_reference_definition():
    # The first draw of SplitMix64::new(0) is the classic splitmix64(0)
    # vector; later draws chain on the mixed state (src/az.rs:3157-3176).
    lib = _lib.lib()
    st = C.c_uint64(0)
    first = lib.cnnue_splitmix64_next(C.byref(st))
    assert first == 0xE220A8397B1DCDAF
    assert st.value == first

    def mix(v):
        m64 = (1 << 64) - 1
        v = (v + 0x9E3779B97F4A7C15) & m64
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m64
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m64
        return v ^ (v >> 31)

    second = lib.cnnue_splitmix64_next(C.byref(st))
    assert second == mix(first)


def test_generators_are_deterministic():
    a = synth.positions(100, 5)
    b = synth.positions(100, 5)
    np.testing.assert_array_equal(a.indices, b.indices)
    c = synth.positions(100, 6)
    assert not np.array_equal(a.indices[:50], c.indices[:50])
    u1 = synth.update_batch(50, 1)
    u2 = synth.update_batch(50, 1)
    np.testing.assert_array_equal(u1.add, u2.add)
    assert u1.flags.max() <= 1 and u1.count0.max() <= 34
