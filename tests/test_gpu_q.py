"""GPU parity of the quantised evaluator (cnnue_q_*) against the oracle:
bit-exact scores and accumulators, golden fixtures, full-size batches and the
edge cases (empty lists, wraparound, every bucket, bad input)."""
import hashlib
import os

import numpy as np
import pytest
import torch

import oracle
from chineseai_b200 import synth
from chineseai_b200._lib import CnnueError
from chineseai_b200.quantized import QuantizedNnue, as_device

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_golden_batch(qmodel):
    g = np.load(GOLDEN)
    pos = synth.Positions(g["q_idx"], g["q_off"])
    scores, acc = qmodel.forward_positions(pos, with_acc=True)
    np.testing.assert_array_equal(scores, g["q_scores"])
    assert sha(acc) == str(g["q_acc_sha"])


@pytest.mark.parametrize("n,seed", [(1, 3), (7, 4), (333, 5), (5000, 6)])
def test_random_batches_bit_exact(qmodel, qweights, n, seed):
    pos = synth.positions(n, seed)
    scores, acc = qmodel.forward_positions(pos, with_acc=True)
    st, ref_scores, ref_acc = oracle.q_forward(qweights, pos, with_acc=True)
    assert st == 0
    np.testing.assert_array_equal(acc, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)


def test_full_batch_65536_bit_exact(qmodel, qweights):
    pos = synth.positions(65536, 1)
    scores, _ = qmodel.forward_positions(pos)
    st, ref = oracle.q_forward_mt(qweights, pos, 0)
    assert st == 0
    np.testing.assert_array_equal(scores, ref)


def test_two_stage_api_and_host_api_agree(qmodel):
    pos = synth.positions(4096, 9)
    ref, _ = qmodel.forward_positions(pos)
    host = qmodel.forward_host(pos.indices, pos.offsets)
    np.testing.assert_array_equal(host, ref)
    # separate bucket sort + sorted forward
    from chineseai_b200._lib import check, lib
    dev = qmodel.device
    idx, off = as_device(pos.indices, dev), as_device(pos.offsets, dev)
    out = torch.empty(pos.n, dtype=torch.int32, device=dev)
    ws = qmodel.workspace(pos.n)
    s = torch.cuda.current_stream().cuda_stream
    check(lib().cnnue_q_bucket_sort(qmodel.handle, off.data_ptr(), len(pos.indices), pos.n, ws.data_ptr(),
                                    ws.numel(), s), "sort")
    check(lib().cnnue_q_forward_sorted(qmodel.handle, idx.data_ptr(), len(pos.indices), off.data_ptr(), pos.n,
                                       out.data_ptr(), ws.data_ptr(), ws.numel(), s), "fwd")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_every_bucket_and_empty_lists(qmodel, qweights):
    # perspective-0 counts 0..40 cover all 16 buckets and the clamp; lists of
    # perspective 1 alternate empty / long.
    rng = np.random.default_rng(1)
    idx, off = [], [0]
    for n0 in range(0, 41):
        for s in range(2):
            k = n0 if s == 0 else (0 if n0 % 2 else 45)
            idx += list(np.sort(rng.choice(11340, size=k, replace=False)))
            off.append(len(idx))
    pos = synth.Positions(np.array(idx, np.uint16), np.array(off, np.uint32))
    scores, acc = qmodel.forward_positions(pos, with_acc=True)
    st, ref_scores, ref_acc = oracle.q_forward(qweights, pos, with_acc=True)
    assert st == 0
    np.testing.assert_array_equal(acc, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)


def test_int16_wraparound(qmodel, qweights):
    idx = np.concatenate([np.full(300, 5, np.uint16), np.full(257, 11339, np.uint16)])
    pos = synth.Positions(idx, np.array([0, 300, 557], np.uint32))
    scores, acc = qmodel.forward_positions(pos, with_acc=True)
    st, ref_scores, ref_acc = oracle.q_forward(qweights, pos, with_acc=True)
    np.testing.assert_array_equal(acc, ref_acc)
    np.testing.assert_array_equal(scores, ref_scores)


def test_empty_batch(qmodel):
    pos = synth.Positions(np.zeros(0, np.uint16), np.zeros(1, np.uint32))
    out = qmodel.forward_host(np.zeros(1, np.uint16), np.zeros(1, np.uint32))
    assert out.shape == (0,)
    assert pos.n == 0


def test_bad_index_and_offsets_are_reported(qmodel, qweights):
    pos = synth.Positions(np.array([3, 11340, 7, 9], np.uint16), np.array([0, 2, 4], np.uint32))
    with pytest.raises(CnnueError) as e:
        qmodel.forward_positions(pos)
    assert e.value.status == 2
    badoff = synth.Positions(np.array([3, 4, 5], np.uint16), np.array([0, 3, 2], np.uint32))
    with pytest.raises(CnnueError) as e:
        qmodel.forward_positions(badoff)
    assert e.value.status == 3
    # the model is still usable afterwards
    good = synth.positions(10, 2)
    scores, _ = qmodel.forward_positions(good)
    np.testing.assert_array_equal(scores, oracle.q_forward(qweights, good)[1])


def test_deterministic_and_stream_safe(qmodel):
    pos = synth.positions(20000, 12)
    a, _ = qmodel.forward_positions(pos)
    s = torch.cuda.Stream()
    idx, off = as_device(pos.indices, qmodel.device), as_device(pos.offsets, qmodel.device)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        out = qmodel.forward(idx, off, pos.n, stream=s)
    s.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), a)


def test_update_golden_and_random(qmodel, qweights):
    g = np.load(GOLDEN)
    ub = synth.UpdateBatch(g["u_parent"], g["u_flags"], g["u_rem"], g["u_rem_offsets"], g["u_add"],
                           g["u_add_offsets"], g["u_count0"])
    child, scores = qmodel.update(ub)
    np.testing.assert_array_equal(scores, g["u_scores"])
    assert sha(child) == str(g["u_child_sha"])
    ub = synth.update_batch(6000, 21)
    child, scores = qmodel.update(ub)
    st, ref_child, ref_scores = oracle.q_update(qweights, ub, 4)
    assert st == 0
    np.testing.assert_array_equal(child, ref_child)
    np.testing.assert_array_equal(scores, ref_scores)


def test_update_full_batch_65536(qmodel, qweights):
    ub = synth.update_batch(65536, 1)
    child, scores = qmodel.update(ub)
    st, ref_child, ref_scores = oracle.q_update(qweights, ub, 0 or oracle.max_threads())
    assert st == 0
    np.testing.assert_array_equal(scores, ref_scores)
    np.testing.assert_array_equal(child, ref_child)


def test_second_model_on_same_device(qweights):
    m2 = QuantizedNnue(qweights, device=0)
    pos = synth.positions(100, 30)
    scores, _ = m2.forward_positions(pos)
    np.testing.assert_array_equal(scores, oracle.q_forward(qweights, pos)[1])
    m2.close()


@pytest.mark.parametrize("n,block,stage", [(64, 0, 0), (64, 5, 1), (3000, 7, 9)])
def test_bounded_wait_runs_out_and_model_recovers(qmodel, qweights, n, block, stage):
    """One CTA leaves one pipeline stage unannounced (nothing copies into it),
    so the consumers' bounded wait on it runs out after 2 ms: the call
    reports CNNUE_ERR_TIMEOUT through the status word, and the next call on
    the same model and workspace is bit-exact again."""
    import ctypes as C

    from chineseai_b200._lib import lib
    pos = synth.positions(n, 40 + block)
    dev = qmodel.device
    idx, off = as_device(pos.indices, dev), as_device(pos.offsets, dev)
    out = torch.empty(pos.n, dtype=torch.int32, device=dev)
    ws = qmodel.workspace(pos.n)
    s = torch.cuda.current_stream().cuda_stream
    rc = lib().cnnue_q_forward_stall_test(qmodel.handle, idx.data_ptr(), len(pos.indices), off.data_ptr(), pos.n,
                                          out.data_ptr(), ws.data_ptr(), ws.numel(), block, stage, 2_000_000, s)
    assert rc == 0
    st = C.c_int(-1)
    assert lib().cnnue_read_status(ws.data_ptr(), s, C.byref(st)) == 0
    assert st.value == 9  # CNNUE_ERR_TIMEOUT
    # the same call without a stall, then the plain forward: both bit-exact
    rc = lib().cnnue_q_forward_stall_test(qmodel.handle, idx.data_ptr(), len(pos.indices), off.data_ptr(), pos.n,
                                          out.data_ptr(), ws.data_ptr(), ws.numel(), 0xFFFFFFFF, 0xFFFFFFFF,
                                          2_000_000, s)
    assert rc == 0
    assert lib().cnnue_read_status(ws.data_ptr(), s, C.byref(st)) == 0 and st.value == 0
    ref = oracle.q_forward(qweights, pos)[1]
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    scores, _ = qmodel.forward_positions(pos)
    np.testing.assert_array_equal(scores, ref)


def test_pipelined_host_contexts(qmodel, qweights):
    """cnnue_q_ctx_*: batches submitted two at a time through one context match
    the device-resident forward bit for bit; a batch with a bad index reports
    it through its own ticket only; a third call in flight is refused; two
    threads with their own contexts share the model."""
    import threading

    from chineseai_b200._lib import CnnueError
    batches = [synth.positions(n, 60 + k) for k, n in enumerate([4096, 1, 3000, 4096, 777])]
    refs = [qmodel.forward_positions(b)[0] for b in batches]
    pinned = lambda a: torch.from_numpy(a).pin_memory().numpy()  # noqa: E731
    pipe = qmodel.pipeline(4096, 4096 * 64)
    outs = [pinned(np.full(b.n, -7, np.int32)) for b in batches]
    tickets = []
    for k, b in enumerate(batches):
        if len(tickets) == 2:
            assert pipe.wait(tickets.pop(0)) == 0
        tickets.append(pipe.submit(pinned(b.indices), pinned(b.offsets), outs[k]))
    for t in tickets:
        assert pipe.wait(t) == 0
    for o, r in zip(outs, refs):
        np.testing.assert_array_equal(o, r)
    # a bad index in one batch: only its ticket reports it
    bad = synth.positions(100, 70)
    bad_idx = bad.indices.copy()
    bad_idx[5] = 11340
    good = batches[2]
    o1, o2 = np.zeros(100, np.int32), np.zeros(good.n, np.int32)
    t1 = pipe.submit(bad_idx, bad.offsets, o1)
    t2 = pipe.submit(good.indices, good.offsets, o2)
    with pytest.raises(CnnueError):
        pipe.submit(good.indices, good.offsets, np.zeros(good.n, np.int32))
    assert pipe.wait(t1) == 2  # CNNUE_ERR_BAD_INDEX
    assert pipe.wait(t2) == 0
    np.testing.assert_array_equal(o2, refs[2])
    pipe.close()

    errors = []

    def worker(seed):
        try:
            p = qmodel.pipeline(2048, 2048 * 64)
            for j in range(3):
                b = synth.positions(2048, seed + j)
                o = np.zeros(b.n, np.int32)
                assert p.wait(p.submit(b.indices, b.offsets, o)) == 0
                np.testing.assert_array_equal(o, oracle.q_forward(qweights, b)[1])
            p.close()
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(100 * i,)) for i in range(2)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
