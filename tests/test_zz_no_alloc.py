"""GPU test of cnnue_q_forward_noalloc, the forward entry point that allocates
nothing (its scratch is a fixed array inside the library).

It exists for callers that cannot allocate device memory while they evaluate:
a search thread that must not stall on cudaMalloc, or a process whose device
memory all belongs to its own pool.  The test calls it through the C ABI, twice
in a row on different batches (the second call must not see the first call's
leftovers in the shared scratch), and compares each result bit for bit with
the regular workspace-taking entry point, cnnue_q_forward.  It also checks that
a batch above the scratch's limit is refused.  This file is collected last so
that a failure here does not hide the other GPU tests.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from chineseai_b200 import synth
from chineseai_b200._lib import check, lib, last_error
from chineseai_b200.quantized import QuantizedNnue, as_device

pytestmark = pytest.mark.gpu

MAX_POSITIONS = 65536


def _with_workspace(model, idx, off, n):
    out = torch.empty(n, dtype=torch.int32, device=model.device)
    ws = torch.empty(model.workspace_bytes(n), dtype=torch.uint8, device=model.device)
    stream = torch.cuda.current_stream().cuda_stream
    check(lib().cnnue_q_forward(model.handle, idx.data_ptr(), idx.numel(), off.data_ptr(), n,
                                out.data_ptr(), ws.data_ptr(), ws.numel(), stream), "cnnue_q_forward")
    st = C.c_int(0)
    check(lib().cnnue_read_status(ws.data_ptr(), stream, C.byref(st)), "cnnue_read_status")
    check(st.value, "cnnue_q_forward (kernel status)")
    return out.cpu().numpy()


def _no_alloc(model, idx, off, n):
    out = torch.empty(n, dtype=torch.int32, device=model.device)
    torch.cuda.synchronize(model.device)
    check(lib().cnnue_q_forward_noalloc(model.handle, idx.data_ptr(), idx.numel(), off.data_ptr(), n,
                                        out.data_ptr(), torch.cuda.current_stream().cuda_stream),
          "cnnue_q_forward_noalloc")
    return out.cpu().numpy()


def test_no_alloc_matches_workspace_entry_point_on_two_calls(qweights):
    model = QuantizedNnue(qweights, device=0)
    try:
        # first call at the limit, second call smaller on other positions
        for n, seed in ((MAX_POSITIONS, 41), (3001, 42)):
            pos = synth.positions(n, seed)
            idx = as_device(pos.indices, model.device)
            off = as_device(pos.offsets, model.device)
            expected = _with_workspace(model, idx, off, n)
            got = _no_alloc(model, idx, off, n)
            np.testing.assert_array_equal(got, expected)
    finally:
        model.close()


def test_no_alloc_refuses_batches_above_its_limit(qweights):
    model = QuantizedNnue(qweights, device=0)
    try:
        n = MAX_POSITIONS + 1
        dummy = torch.zeros(2 * n + 1, dtype=torch.int32, device=model.device)
        out = torch.empty(n, dtype=torch.int32, device=model.device)
        st = lib().cnnue_q_forward_noalloc(model.handle, dummy.data_ptr(), 0, dummy.data_ptr(), n,
                                           out.data_ptr(), None)
        assert st == 1  # CNNUE_ERR_INVALID_ARG
        assert str(MAX_POSITIONS) in last_error()
    finally:
        model.close()


def test_no_alloc_allocates_nothing_and_clears_its_status(qweights):
    """The property the entry point exists for: once the library and the
    model are set up (a first call has looked up the scratch address), a call
    takes no device memory - the device's free memory is the same after it.
    A call on bad offsets reports CNNUE_ERR_BAD_OFFSETS through the shared
    scratch's status word, and the next good call is clean and exact."""
    model = QuantizedNnue(qweights, device=0)
    try:
        pos = synth.positions(4096, 43)
        idx = as_device(pos.indices, model.device)
        off = as_device(pos.offsets, model.device)
        expected = _with_workspace(model, idx, off, pos.n)
        out = torch.empty(pos.n, dtype=torch.int32, device=model.device)
        stream = torch.cuda.current_stream().cuda_stream
        call = lambda i, o, n: lib().cnnue_q_forward_noalloc(  # noqa: E731
            model.handle, i.data_ptr(), i.numel(), o.data_ptr(), n, out.data_ptr(), stream)
        assert call(idx, off, pos.n) == 0  # warm-up: the scratch address is looked up here
        torch.cuda.synchronize()
        free_before, _ = torch.cuda.mem_get_info(model.device)
        for _ in range(3):
            assert call(idx, off, pos.n) == 0
        torch.cuda.synchronize()
        free_after, _ = torch.cuda.mem_get_info(model.device)
        assert free_after == free_before
        np.testing.assert_array_equal(out.cpu().numpy(), expected)
        bad_idx = as_device(np.array([3, 4, 5], np.uint16), model.device)
        bad_off = as_device(np.array([0, 3, 2], np.uint32), model.device)
        assert call(bad_idx, bad_off, 1) == 3  # CNNUE_ERR_BAD_OFFSETS
        assert call(idx, off, pos.n) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), expected)
    finally:
        model.close()
