"""CPU oracle of the NNUE hot path - TEST INFRASTRUCTURE ONLY.

ctypes wrapper of oracle/liboracle.so (built from cnnue_oracle.c by
oracle/Makefile).  Only tests/, the smoke check and bench.py's CPU-baseline
leg use it, always as the checker; the product library never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or (
                os.path.getmtime(os.path.join(HERE, "cnnue_oracle.c")) > os.path.getmtime(LIB_PATH)):
            build()
        h = C.CDLL(LIB_PATH)
        P, i64, u32, i32 = C.c_void_p, C.c_int64, C.c_uint32, C.c_int
        h.oracle_q_forward.argtypes = [P] * 9 + [u32, P, i64, P, P]
        h.oracle_q_forward_mt.argtypes = [P] * 9 + [u32, P, i64, P, i32]
        h.oracle_q_update.argtypes = [P] * 10 + [P, u32, P, P, u32, P, P, i64, P, P, i32]
        h.oracle_f_forward.argtypes = [P] * 9 + [u32, P, i64, P, P]
        h.oracle_feature_pool_fwd.argtypes = [P, P, i64, i64, i64, P]
        h.oracle_feature_pool_bwd.argtypes = [P, P, i64, i64, i64, P]
        h.oracle_sparse_pool_fwd.argtypes = [P, i64, P, i64, i64, i64, P]
        h.oracle_sparse_pool_bwd.argtypes = [P, P, i64, i64, i64, i64, P]
        h.oracle_policy_fused_fwd.argtypes = [P, P, P, i64, i64, P]
        h.oracle_policy_fused_bwd.argtypes = [P, P, P, P, i64, i64, P, P]
        h.oracle_policy_table_fwd.argtypes = [P, i64, P, i64, i32, P]
        h.oracle_policy_table_bwd.argtypes = [P, P, i64, i32, i64, P]
        h.oracle_adamw.argtypes = [P, P, P, P, i64, C.c_double, C.c_double, C.c_double, C.c_double,
                                    C.c_double, i64]
        h.oracle_q_bucket.argtypes = [u32]
        h.oracle_f_bucket.argtypes = [u32]
        for name in ("oracle_q_forward", "oracle_q_forward_mt", "oracle_q_update", "oracle_f_forward",
                     "oracle_feature_pool_fwd", "oracle_feature_pool_bwd", "oracle_sparse_pool_fwd",
                     "oracle_sparse_pool_bwd", "oracle_q_bucket", "oracle_f_bucket",
                     "oracle_policy_fused_fwd", "oracle_policy_fused_bwd", "oracle_policy_table_fwd",
                     "oracle_policy_table_bwd", "oracle_adamw",
                     "oracle_max_threads"):
            getattr(h, name).restype = C.c_int
        _lib = h
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def q_forward(w, pos, with_acc: bool = False):
    """Quantised forward -> (status, scores int32[n], acc int16[n,2,1024] | None)."""
    n = pos.n
    scores = np.zeros(max(n, 1), np.int32)
    acc = np.zeros((max(n, 1), 2, 1024), np.int16) if with_acc else None
    arrs = w.arrays()
    idx = pos.indices if len(pos.indices) else np.zeros(1, np.uint16)
    st = lib().oracle_q_forward(*[_p(a) for a in arrs], _p(idx), len(pos.indices), _p(pos.offsets), n,
                                _p(scores), _p(acc) if with_acc else None)
    return st, scores[:n], (acc[:n] if with_acc else None)


def q_forward_mt(w, pos, n_threads: int = 0):
    n = pos.n
    scores = np.zeros(max(n, 1), np.int32)
    st = lib().oracle_q_forward_mt(*[_p(a) for a in w.arrays()], _p(pos.indices), len(pos.indices),
                                   _p(pos.offsets), n, _p(scores), n_threads)
    return st, scores[:n]


def q_update(w, batch, n_threads: int = 1):
    n = batch.n
    child = np.zeros((max(n, 1), 2, 1024), np.int16)
    scores = np.zeros(max(n, 1), np.int32)
    rem = batch.rem if len(batch.rem) else np.zeros(1, np.uint16)
    add = batch.add if len(batch.add) else np.zeros(1, np.uint16)
    st = lib().oracle_q_update(*[_p(a) for a in w.arrays()], _p(batch.parent), _p(batch.flags), _p(rem),
                               len(batch.rem), _p(batch.rem_offsets), _p(add), len(batch.add),
                               _p(batch.add_offsets), _p(batch.count0), n, _p(child), _p(scores),
                               n_threads)
    return st, child[:n], scores[:n]


def f_forward(w, pos, with_acc: bool = False):
    n = pos.n
    out = np.zeros(max(n, 1), np.float32)
    acc = np.zeros((max(n, 1), 2, 256), np.float32) if with_acc else None
    idx = pos.indices if len(pos.indices) else np.zeros(1, np.uint16)
    st = lib().oracle_f_forward(*[_p(a) for a in w.arrays()], _p(idx), len(pos.indices), _p(pos.offsets),
                                n, _p(out), _p(acc) if with_acc else None)
    return st, out[:n], (acc[:n] if with_acc else None)


def feature_pool_fwd(tables: np.ndarray, items: np.ndarray, hidden: int):
    batch, item_count = items.shape
    out = np.zeros((batch, hidden), np.float32)
    st = lib().oracle_feature_pool_fwd(_p(tables), _p(items), batch, item_count, hidden, _p(out))
    return st, out


def feature_pool_bwd(items: np.ndarray, grad_out: np.ndarray, hidden: int):
    batch, item_count = items.shape
    grad = np.zeros((1545, hidden), np.float32)
    st = lib().oracle_feature_pool_bwd(_p(items), _p(grad_out), batch, item_count, hidden, _p(grad))
    return st, grad


def sparse_pool_fwd(table: np.ndarray, items: np.ndarray):
    rows, hidden = table.shape
    batch, item_count = items.shape
    out = np.zeros((batch, hidden), np.float32)
    st = lib().oracle_sparse_pool_fwd(_p(table), rows, _p(items), batch, item_count, hidden, _p(out))
    return st, out


def sparse_pool_bwd(items: np.ndarray, grad_out: np.ndarray, rows: int):
    batch, item_count = items.shape
    hidden = grad_out.shape[1]
    grad = np.zeros((rows, hidden), np.float32)
    st = lib().oracle_sparse_pool_bwd(_p(items), _p(grad_out), rows, batch, item_count, hidden, _p(grad))
    return st, grad


POLICY_TABLE_LEN = 182886
POLICY_CONTEXT = 48


def policy_fused_fwd(tables: np.ndarray, context: np.ndarray, items: np.ndarray):
    """FusedPolicy forward restated -> (status, logits [B][M])."""
    batch, moves = items.shape
    out = np.zeros((max(batch, 1), max(moves, 1)), np.float32)
    st = lib().oracle_policy_fused_fwd(_p(np.ascontiguousarray(tables, np.float32)),
                                       _p(np.ascontiguousarray(context, np.float32)),
                                       _p(np.ascontiguousarray(items, np.int64)), batch, moves, _p(out))
    return st, out[:batch, :moves]


def policy_fused_bwd(tables: np.ndarray, context: np.ndarray, items: np.ndarray, grad_out: np.ndarray):
    """FusedPolicyGrad restated -> (status, grad_tables [182886], grad_context [B][48])."""
    batch, moves = items.shape
    gt = np.zeros(POLICY_TABLE_LEN, np.float32)
    gc = np.zeros((max(batch, 1), POLICY_CONTEXT), np.float32)
    st = lib().oracle_policy_fused_bwd(_p(np.ascontiguousarray(tables, np.float32)),
                                       _p(np.ascontiguousarray(context, np.float32)),
                                       _p(np.ascontiguousarray(items, np.int64)),
                                       _p(np.ascontiguousarray(grad_out, np.float32)), batch, moves, _p(gt),
                                       _p(gc))
    return st, gt, gc[:batch]


def policy_table_fwd(table: np.ndarray, indices: np.ndarray):
    """SparsePolicy forward restated; indices [..., terms] -> (status, out [...])."""
    terms = indices.shape[-1]
    flat = np.ascontiguousarray(indices, np.int64).reshape(-1, terms)
    out = np.zeros(max(len(flat), 1), np.float32)
    st = lib().oracle_policy_table_fwd(_p(np.ascontiguousarray(table, np.float32)), len(table), _p(flat),
                                       len(flat), terms, _p(out))
    return st, out[:len(flat)].reshape(indices.shape[:-1])


def policy_table_bwd(indices: np.ndarray, grad_out: np.ndarray, table_len: int):
    """SparsePolicyGrad restated -> (status, grad_table [table_len])."""
    terms = indices.shape[-1]
    flat = np.ascontiguousarray(indices, np.int64).reshape(-1, terms)
    g = np.ascontiguousarray(grad_out, np.float32).reshape(-1)
    grad = np.zeros(table_len, np.float32)
    st = lib().oracle_policy_table_bwd(_p(flat), _p(g), len(flat), terms, table_len, _p(grad))
    return st, grad


def adamw(p, m, v, g, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-4, step=1):
    """candle-nn AdamW step restated, in place on float32 arrays p, m, v."""
    for a in (p, m, v):
        assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    g = np.ascontiguousarray(g, np.float32)
    return lib().oracle_adamw(_p(p), _p(m), _p(v), _p(g), p.size, lr, beta1, beta2, eps, weight_decay, step)


def q_bucket(n0: int) -> int:
    return lib().oracle_q_bucket(n0)


def max_threads() -> int:
    return lib().oracle_max_threads()


def _t_setup(h):
    if getattr(h, "_t_ready", False):
        return
    P, i64, u32, i32, f32 = C.c_void_p, C.c_int64, C.c_uint32, C.c_int, C.c_float
    h.oracle_t_grad.argtypes = [P] * 9 + [u32, P, i64, P] + [P] * 8 + [P, P]
    h.oracle_t_grad.restype = C.c_int
    h.oracle_adam.argtypes = [P, P, P, P, i64, f32, f32, f32, f32, f32, i32]
    h.oracle_adam.restype = None
    h.oracle_bf16_round_array.argtypes = [P, P, i64]
    h.oracle_bf16_round_array.restype = None
    h._t_ready = True


def t_grad(params: np.ndarray, pos, target: np.ndarray):
    """Training-step gradients of one rank's batch: (status, loss, flat grads)."""
    from chineseai_b200.train import LAYOUT, split
    h = lib()
    _t_setup(h)
    p = split(np.ascontiguousarray(params, np.float32))
    g_flat = np.zeros_like(params, dtype=np.float32)
    g = split(g_flat)
    loss = C.c_float(0.0)
    idx = pos.indices if len(pos.indices) else np.zeros(1, np.uint16)
    tgt = np.ascontiguousarray(target, np.float32)
    st = h.oracle_t_grad(*[_p(np.ascontiguousarray(p[n])) for n, _ in LAYOUT], _p(idx), len(pos.indices),
                         _p(pos.offsets), pos.n, _p(tgt), *[_p(g[n]) for n, _ in LAYOUT], C.byref(loss), None)
    return st, loss.value, g_flat


def adam(w: np.ndarray, m: np.ndarray, v: np.ndarray, g: np.ndarray, grad_scale: float, lr: float,
         beta1: float, beta2: float, eps: float, step: int) -> None:
    h = lib()
    _t_setup(h)
    h.oracle_adam(_p(w), _p(m), _p(v), _p(g), len(w), grad_scale, lr, beta1, beta2, eps, step)


def bf16_round(a: np.ndarray) -> np.ndarray:
    h = lib()
    _t_setup(h)
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty_like(a)
    h.oracle_bf16_round_array(_p(a), _p(out), a.size)
    return out


# ---- AZ-NNUE (reference-native) ---------------------------------------------
def _az_setup(h):
    if getattr(h, "_az_ready", False):
        return
    P, i64, i32, u64 = C.c_void_p, C.c_int64, C.c_int, C.c_uint64
    h.oracle_az_tensor_elements.argtypes = [i32, i32]
    h.oracle_az_tensor_elements.restype = i64
    h.oracle_az_random.argtypes = [i32, u64, P]
    h.oracle_az_random.restype = None
    h.oracle_az_features.argtypes = [P, i32, P]
    h.oracle_az_features.restype = i32
    h.oracle_az_refresh.argtypes = [P, P, i32, P, P, i64, P]
    h.oracle_az_refresh.restype = i32
    h.oracle_az_transition.argtypes = [P, P, i32, P, P, P, P, P, i64, P]
    h.oracle_az_transition.restype = i32
    h.oracle_az_value.argtypes = [P, P, P, P, i32, P, P, P, i64, P, P, P]
    h.oracle_az_value.restype = None
    h._az_ready = True


def _az():
    h = lib()
    _az_setup(h)
    return h


def az_random(hidden: int, seed: int):
    """AzNnue::random(hidden, seed) restated: the 22 tensors, flat float32."""
    h = _az()
    arrays = [np.zeros(h.oracle_az_tensor_elements(i, hidden), np.float32) for i in range(22)]
    ptrs = (C.c_void_p * 22)(*[a.ctypes.data for a in arrays])
    h.oracle_az_random(hidden, seed, ptrs)
    return arrays


def az_features(board: np.ndarray, perspective: int) -> np.ndarray:
    items = np.zeros(90, np.uint32)
    b = np.ascontiguousarray(board, np.int8)
    n = _az().oracle_az_features(_p(b), perspective, _p(items))
    return items[:n].copy()


def az_trunk(tensors) -> tuple:
    """(trunk [1545][H], bias [H]) from the 22 tensors."""
    trunk = np.ascontiguousarray(np.concatenate([np.asarray(tensors[i], np.float32).reshape(-1) for i in range(5)]))
    return trunk, np.ascontiguousarray(np.asarray(tensors[6], np.float32).reshape(-1))


def az_refresh(tensors, hidden: int, items: np.ndarray, offsets: np.ndarray):
    trunk, bias = az_trunk(tensors)
    n_lists = len(offsets) - 1
    acc = np.zeros((max(n_lists, 1), hidden), np.float32)
    it = np.ascontiguousarray(items, np.uint32) if len(items) else np.zeros(1, np.uint32)
    st = _az().oracle_az_refresh(_p(trunk), _p(bias), hidden, _p(it), _p(np.ascontiguousarray(offsets, np.uint32)),
                                 n_lists, _p(acc))
    return st, acc[:n_lists]


def az_transition(tensors, hidden: int, parent: np.ndarray, delta: np.ndarray, refresh: np.ndarray,
                  items: np.ndarray, offsets: np.ndarray):
    trunk, bias = az_trunk(tensors)
    n_lists = len(refresh)
    child = np.zeros((max(n_lists, 1), hidden), np.float32)
    it = np.ascontiguousarray(items, np.uint32) if len(items) else np.zeros(1, np.uint32)
    st = _az().oracle_az_transition(_p(trunk), _p(bias), hidden, _p(np.ascontiguousarray(parent, np.float32)),
                                    _p(np.ascontiguousarray(delta, np.uint32)),
                                    _p(np.ascontiguousarray(refresh, np.uint8)), _p(it),
                                    _p(np.ascontiguousarray(offsets, np.uint32)), n_lists, _p(child))
    return st, child[:n_lists]


def az_value(tensors, hidden: int, hidden_rows: np.ndarray, rule=None, threat=None, with_x: bool = False):
    """(wdl [n][3], q [n]) from side-to-move accumulators [n][H]; with_x adds
    the normalised hidden [n][H] the policy head reads."""
    n = hidden_rows.shape[0]
    wdl = np.zeros((max(n, 1), 3), np.float32)
    q = np.zeros(max(n, 1), np.float32)
    x = np.zeros((max(n, 1), hidden), np.float32) if with_x else None
    f = [np.ascontiguousarray(np.asarray(tensors[i], np.float32).reshape(-1)) for i in (5, 7, 8, 9)]
    r = None if rule is None else np.ascontiguousarray(rule, np.float32)
    t = None if threat is None else np.ascontiguousarray(threat, np.float32)
    _az().oracle_az_value(_p(f[0]), _p(f[1]), _p(f[2]), _p(f[3]), hidden,
                          _p(np.ascontiguousarray(hidden_rows, np.float32)), None if r is None else _p(r),
                          None if t is None else _p(t), n, _p(wdl), _p(q), _p(x) if with_x else None)
    if with_x:
        return wdl[:n], q[:n], x[:n]
    return wdl[:n], q[:n]


def _azq_setup(h):
    if getattr(h, "_azq_ready", False):
        return
    P, i64, i32 = C.c_void_p, C.c_int64, C.c_int
    h.oracle_az_dense_moves.argtypes = [P]
    h.oracle_az_dense_moves.restype = i32
    h.oracle_az_quantize.argtypes = [i32, P] + [P] * 8
    h.oracle_az_quantize.restype = i32
    h.oracle_az_policy_refresh.argtypes = [P, P, P, i64, P]
    h.oracle_az_policy_refresh.restype = i32
    h.oracle_az_policy_transition.argtypes = [P, P, P, P, P, P, i64, P]
    h.oracle_az_policy_transition.restype = i32
    h._azq_ready = True


def _azq():
    h = _az()
    _azq_setup(h)
    return h


def az_dense_moves() -> np.ndarray:
    out = np.zeros(8100, np.uint16)
    n = _azq().oracle_az_dense_moves(_p(out))
    return out[:n].copy()


def az_quantize(tensors, hidden: int) -> dict:
    """rebuild_policy_accumulator_quantization + rebuild_value_threat_quantization restated."""
    flat = [np.ascontiguousarray(np.asarray(t, np.float32).reshape(-1)) for t in tensors]
    ptrs = (C.c_void_p * 22)(*[a.ctypes.data for a in flat])
    out = {"policy_feature": np.zeros((1546, 32), np.int8), "policy_move": np.zeros((2086, 32), np.int8),
           "policy_sparse": np.zeros(2396815, np.int8), "moved_delta": np.zeros((2086, 14), np.int32),
           "capture": np.zeros((2086, 14), np.int32), "value_threat": np.zeros((57702, 64), np.int8)}
    scales = np.zeros(4, np.float32)
    flags = np.zeros(2, np.int32)
    st = _azq().oracle_az_quantize(hidden, ptrs, *[_p(out[k]) for k in ("policy_feature", "policy_move",
                                                                        "policy_sparse", "moved_delta", "capture",
                                                                        "value_threat")], _p(scales), _p(flags))
    assert st == 0
    out["scales"] = scales
    out["flags"] = flags
    return out


def az_policy_refresh(feature_q: np.ndarray, items: np.ndarray, offsets: np.ndarray):
    n_lists = len(offsets) - 1
    acc = np.zeros((max(n_lists, 1), 32), np.int16)
    it = np.ascontiguousarray(items, np.uint32) if len(items) else np.zeros(1, np.uint32)
    st = _azq().oracle_az_policy_refresh(_p(np.ascontiguousarray(feature_q, np.int8)), _p(it),
                                         _p(np.ascontiguousarray(offsets, np.uint32)), n_lists, _p(acc))
    return st, acc[:n_lists]


def az_policy_transition(feature_q, parent, delta, refresh, items, offsets):
    n_lists = len(refresh)
    child = np.zeros((max(n_lists, 1), 32), np.int16)
    it = np.ascontiguousarray(items, np.uint32) if len(items) else np.zeros(1, np.uint32)
    st = _azq().oracle_az_policy_transition(_p(np.ascontiguousarray(feature_q, np.int8)),
                                            _p(np.ascontiguousarray(parent, np.int16)),
                                            _p(np.ascontiguousarray(delta, np.uint32)),
                                            _p(np.ascontiguousarray(refresh, np.uint8)), _p(it),
                                            _p(np.ascontiguousarray(offsets, np.uint32)), n_lists, _p(child))
    return st, child[:n_lists]


def rn_forward(weights, planes_bits: np.ndarray, with_trunk: bool = False):
    """ResNet forward restated on the CPU: (logits, probs, value_pre, value, trunk|None)."""
    h = lib()
    if not getattr(h, "_rn_ready", False):
        h.oracle_rn_forward.argtypes = [C.c_void_p] * 15 + [C.c_int64] + [C.c_void_p] * 5
        h.oracle_rn_forward.restype = None
        h._rn_ready = True
    B = planes_bits.shape[0]
    planes = np.ascontiguousarray((planes_bits.astype(np.uint32) << 16).view(np.float32).reshape(B, 15, 90))
    arrs = weights.arrays()
    logits = np.zeros((max(B, 1), 2086), np.float32)
    probs = np.zeros((max(B, 1), 2086), np.float32)
    vpre = np.zeros(max(B, 1), np.float32)
    value = np.zeros(max(B, 1), np.float32)
    trunk = np.zeros((max(B, 1), 128, 90), np.float32) if with_trunk else None
    h.oracle_rn_forward(*[_p(a) for a in arrs], _p(planes), B, _p(logits), _p(probs), _p(vpre), _p(value),
                        _p(trunk) if with_trunk else None)
    return logits[:B], probs[:B], vpre[:B], value[:B], (trunk[:B] if with_trunk else None)


def _azt():
    h = _az()
    if not getattr(h, "_azt_ready", False):
        h.oracle_az_threat_vocab.restype = C.c_int
        h.oracle_az_threat_features.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        h.oracle_az_threat_features.restype = C.c_int
        h.oracle_az_threat_logits.argtypes = [C.c_void_p, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p,
                                              C.c_int64, C.c_void_p, C.c_void_p]
        h.oracle_az_policy_moves.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
        h.oracle_az_policy_moves.restype = C.c_int
        h.oracle_az_policy_logits.argtypes = [C.c_void_p, C.c_int] + [C.c_void_p] * 5 + [C.c_int] + \
            [C.c_void_p] * 5 + [C.c_int64, C.c_void_p]
        h.oracle_az_policy_logits.restype = C.c_int
        h.oracle_az_threat_logits.restype = C.c_int
        h._azt_ready = True
    return h


def az_threat_vocab() -> int:
    return _azt().oracle_az_threat_vocab()


def az_threat_features(board: np.ndarray, side: int) -> np.ndarray:
    out = np.zeros(256, np.uint32)
    n = _azt().oracle_az_threat_features(_p(np.ascontiguousarray(board, np.int8)), side, _p(out))
    return out[:n].copy()


def az_threat_logits(table: np.ndarray, scale: float, out_w: np.ndarray, features: np.ndarray, offsets: np.ndarray,
                     with_act: bool = False):
    n = len(offsets) - 1
    logits = np.zeros((max(n, 1), 3), np.float32)
    act = np.zeros((max(n, 1), 128), np.float32) if with_act else None
    f = np.ascontiguousarray(features, np.uint32) if len(features) else np.zeros(1, np.uint32)
    st = _azt().oracle_az_threat_logits(_p(np.ascontiguousarray(table, np.int8)), scale,
                                        _p(np.ascontiguousarray(out_w, np.float32)), _p(f),
                                        _p(np.ascontiguousarray(offsets, np.uint32)), n, _p(logits),
                                        _p(act) if with_act else None)
    if with_act:
        return st, logits[:n], act[:n]
    return st, logits[:n]


def az_policy_moves(board: np.ndarray, side: int, moves: np.ndarray) -> np.ndarray:
    mv = np.ascontiguousarray(moves, np.uint8).reshape(-1, 2)
    info = np.zeros((max(len(mv), 1), 2), np.uint32)
    _azt().oracle_az_policy_moves(_p(np.ascontiguousarray(board, np.int8)), side, _p(mv), len(mv), _p(info))
    return info[:len(mv)]


def az_policy_logits(tensors, hidden: int, quant: dict, tactical_active: bool, x, act, pacc, info, offsets):
    """Per-move policy logits restated (quant = az_quantize's output)."""
    flat = [np.ascontiguousarray(np.asarray(t, np.float32).reshape(-1)) for t in tensors]
    ptrs = (C.c_void_p * 22)(*[a.ctypes.data for a in flat])
    n = len(offsets) - 1
    logits = np.zeros(max(int(offsets[-1]), 1), np.float32)
    _azt().oracle_az_policy_logits(ptrs, hidden, _p(quant["policy_move"]), _p(quant["policy_sparse"]),
                                   _p(quant["moved_delta"]), _p(quant["capture"]),
                                   _p(np.ascontiguousarray(quant["scales"], np.float32)), int(tactical_active),
                                   _p(np.ascontiguousarray(x, np.float32)),
                                   None if act is None else _p(np.ascontiguousarray(act, np.float32)),
                                   _p(np.ascontiguousarray(pacc, np.int16)),
                                   _p(np.ascontiguousarray(info, np.uint32)),
                                   _p(np.ascontiguousarray(offsets, np.uint32)), n, _p(logits))
    return logits[:int(offsets[-1])]
