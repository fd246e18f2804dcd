"""ctypes binding of libcnnue.so (the C ABI declared in include/cnnue.h).

The library is loaded from the package directory only.  When it is missing the
import fails loudly: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libcnnue.so")

c_void_p = C.c_void_p
c_int = C.c_int
c_i64 = C.c_int64
c_u32 = C.c_uint32
c_u64 = C.c_uint64
c_size = C.c_size_t
P = C.c_void_p  # every buffer crosses the ABI as a plain pointer


class QWeights(C.Structure):
    _fields_ = [(n, c_void_p) for n in (
        "ft_weight", "ft_bias", "l1_weight", "l1_bias", "l2_weight", "l2_bias", "l3_weight", "l3_bias")]


class FWeights(C.Structure):
    _fields_ = [(n, c_void_p) for n in (
        "ft_weight", "ft_bias", "l1_weight", "l1_bias", "l2_weight", "l2_bias", "l3_weight", "l3_bias")]


# name -> (restype, argtypes)
SIGNATURES = {
    "cnnue_status_string": (C.c_char_p, [c_int]),
    "cnnue_last_error": (C.c_char_p, []),
    "cnnue_version": (C.c_char_p, []),
    "cnnue_q_model_create": (c_int, [C.POINTER(QWeights), c_int, C.POINTER(c_void_p)]),
    "cnnue_q_model_destroy": (c_int, [c_void_p]),
    "cnnue_q_workspace_bytes": (c_size, [c_i64]),
    "cnnue_read_status": (c_int, [P, P, C.POINTER(c_int)]),
    "cnnue_q_forward": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_q_bucket_sort": (c_int, [c_void_p, P, c_u32, c_i64, P, c_size, P]),
    "cnnue_q_forward_sorted": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_q_forward_host": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P]),
    "cnnue_q_forward_acc": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, P, c_size, P]),
    "cnnue_q_forward_noalloc": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P]),
    "cnnue_q_ctx_create": (c_int, [c_void_p, c_i64, c_u32, C.POINTER(c_void_p)]),
    "cnnue_q_ctx_destroy": (c_int, [c_void_p]),
    "cnnue_q_ctx_next_stream": (c_int, [c_void_p, C.POINTER(c_void_p)]),
    "cnnue_q_forward_host_async": (c_int, [c_void_p, P, c_u32, P, c_i64, P, C.POINTER(c_u64)]),
    "cnnue_q_ctx_wait": (c_int, [c_void_p, c_u64, C.POINTER(c_int)]),
    "cnnue_q_forward_stall_test": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, c_u32, c_u32, c_u64, P]),
    "cnnue_q_update": (c_int, [c_void_p, P, P, P, c_u32, P, P, c_u32, P, P, c_i64, P, P, P,
                               c_size, P]),
    "cnnue_f_model_create": (c_int, [C.POINTER(FWeights), c_int, C.POINTER(c_void_p)]),
    "cnnue_f_model_destroy": (c_int, [c_void_p]),
    "cnnue_f_workspace_bytes": (c_size, [c_i64]),
    "cnnue_f_forward": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_feature_pool_fwd": (c_int, [P, P, c_i64, c_i64, c_i64, P, P, P]),
    "cnnue_feature_pool_bwd_workspace_bytes": (c_size, [c_i64, c_i64, c_i64]),
    "cnnue_feature_pool_bwd": (c_int, [P, P, c_i64, c_i64, c_i64, P, P, c_size, P]),
    "cnnue_sparse_pool_fwd": (c_int, [P, c_i64, P, c_i64, c_i64, c_i64, P, P, P]),
    "cnnue_sparse_pool_bwd_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_i64]),
    "cnnue_sparse_pool_bwd": (c_int, [P, P, c_i64, c_i64, c_i64, c_i64, P, P, c_size, P]),
    "cnnue_policy_fused_fwd": (c_int, [P, P, P, c_i64, c_i64, P, P, P]),
    "cnnue_policy_fused_bwd_workspace_bytes": (c_size, [c_i64, c_i64]),
    "cnnue_policy_fused_bwd": (c_int, [P, P, P, P, c_i64, c_i64, P, P, P, c_size, P]),
    "cnnue_policy_table_fwd": (c_int, [P, c_i64, P, c_i64, c_int, P, P, P]),
    "cnnue_policy_table_bwd_workspace_bytes": (c_size, [c_i64, c_int]),
    "cnnue_policy_table_bwd": (c_int, [P, P, c_i64, c_int, c_i64, P, P, c_size, P]),
    "cnnue_adamw": (c_int, [P, P, P, P, c_i64, C.c_double, C.c_double, C.c_double, C.c_double, C.c_double,
                            c_i64, P]),
    "cnnue_adamw_device": (c_int, [P, P, P, P, c_i64, P, P]),
    "cnnue_adamw_device_scaled": (c_int, [P, P, P, P, c_i64, P, C.c_float, P, c_int, P]),
    "cnnue_t_param_count": (c_size, []),
    "cnnue_t_workspace_bytes": (c_size, [c_i64, c_u32]),
    "cnnue_t_make_shadow": (c_int, [P, P, P]),
    "cnnue_t_forward_backward": (c_int, [P, P, P, c_u32, P, c_i64, P, P, P, P, c_size, P]),
    "cnnue_t_adam": (c_int, [P, P, P, P, P, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float,
                             c_int, P, P]),
    "cnnue_t_adam_range": (c_int, [P, P, P, P, P, c_i64, c_i64, C.c_float, C.c_float, C.c_float, C.c_float,
                                   C.c_float, c_int, P, P]),
    "cnnue_t_forward_backward_begin": (c_int, [P, P, P, c_u32, P, c_i64, P, P, P, c_size, P]),
    "cnnue_t_ft_grad_rows": (c_int, [c_i64, c_u32, P, P, c_size, c_i64, c_i64, P]),
    "cnnue_t_finish": (c_int, [c_i64, c_u32, P, P, c_size, P, P]),
    "cnnue_az_board_from_fen": (c_int, [C.c_char_p, P, C.POINTER(c_int)]),
    "cnnue_az_features": (c_int, [P, c_int, P, C.POINTER(c_int)]),
    "cnnue_az_move_items": (c_int, [P, c_int, c_int, c_int, P, P, P, C.POINTER(c_int)]),
    "cnnue_az_tensor_info": (c_int, [c_int, c_i64, C.POINTER(C.c_char_p), C.POINTER(c_i64)]),
    "cnnue_az_weights_random": (c_int, [c_i64, c_u64, C.POINTER(c_void_p)]),
    "cnnue_az_weights_load": (c_int, [C.c_char_p, C.POINTER(c_void_p)]),
    "cnnue_az_weights_save": (c_int, [c_void_p, C.c_char_p]),
    "cnnue_az_weights_destroy": (c_int, [c_void_p]),
    "cnnue_az_weights_hidden": (c_i64, [c_void_p]),
    "cnnue_az_weights_tensor": (c_int, [c_void_p, c_int, C.POINTER(C.POINTER(C.c_float)), C.POINTER(c_i64)]),
    "cnnue_az_model_create": (c_int, [c_void_p, c_int, C.POINTER(c_void_p)]),
    "cnnue_az_model_destroy": (c_int, [c_void_p]),
    "cnnue_az_model_device": (c_int, [c_void_p]),
    "cnnue_az_workspace_bytes": (c_size, []),
    "cnnue_az_refresh": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_az_transition": (c_int, [c_void_p, P, P, P, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_az_value": (c_int, [c_void_p, P, P, P, P, c_i64, P, P, P]),
    "cnnue_az_quantize": (c_int, [c_void_p]),
    "cnnue_az_quant_table": (c_int, [c_void_p, c_int, C.POINTER(c_void_p), C.POINTER(c_i64),
                                     C.POINTER(C.c_float)]),
    "cnnue_az_quant_flags": (c_int, [c_void_p, C.POINTER(c_int), C.POINTER(c_int)]),
    "cnnue_az_dense_moves": (c_int, [P, P]),
    "cnnue_az_policy_refresh": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_az_policy_transition": (c_int, [c_void_p, P, P, P, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_az_threat_features": (c_int, [P, c_int, P, C.POINTER(c_int)]),
    "cnnue_az_threat_vocab": (c_int, []),
    "cnnue_az_threat_logits": (c_int, [c_void_p, P, c_u32, P, c_i64, P, P, c_size, P]),
    "cnnue_az_policy_moves": (c_int, [P, c_int, P, c_int, P]),
    "cnnue_az_pack_batch": (c_int, [c_void_p, P, c_i64, c_i64, c_i64, c_i64, c_int, c_void_p, c_int]),
    "cnnue_az_expand_policy_indices": (c_int, [P, P, P, c_i64, c_i64, P, P, P, P]),
    "cnnue_azt_create": (c_int, [c_int, C.POINTER(c_void_p)]),
    "cnnue_azt_destroy": (c_int, [c_void_p]),
    "cnnue_azt_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "cnnue_azt_step": (c_int, [c_void_p, P, P, c_i64, P, c_i64, P, C.c_float, C.c_float, P, P, P, c_size, P, P]),
    "cnnue_az_legal_moves": (c_int, [P, c_int, P, c_int, C.POINTER(c_int)]),
    "cnnue_mcts_default_limits": (None, [c_void_p]),
    "cnnue_mcts_create": (c_int, [c_void_p, c_void_p, c_int, C.POINTER(c_void_p)]),
    "cnnue_mcts_destroy": (c_int, [c_void_p]),
    "cnnue_mcts_search": (c_int, [c_void_p, P, P, P, c_i64, c_void_p, P, C.POINTER(c_u64)]),
    "cnnue_mcts_stats": (c_int, [c_void_p, P, C.POINTER(c_u64)]),
    "cnnue_mcts_result": (c_int, [c_void_p, c_i64, P, P, P, P, c_int, C.POINTER(c_int), C.POINTER(c_int),
                                  C.POINTER(C.c_float), C.POINTER(c_u32)]),
    "cnnue_az_evaluate_workspace_bytes": (c_size, [c_void_p, c_i64]),
    "cnnue_az_evaluate": (c_int, [c_void_p, P, P, P, P, c_u32, P, P, P, c_u32, P, c_i64, P, P, P, P, c_size, P]),
    "cnnue_rn_model_create": (c_int, [C.c_void_p, c_int, C.POINTER(c_void_p)]),
    "cnnue_rn_model_destroy": (c_int, [c_void_p]),
    "cnnue_rn_workspace_bytes": (c_size, [c_i64]),
    "cnnue_rn_forward": (c_int, [c_void_p, P, c_i64, P, P, P, P, c_size, P]),
    "cnnue_rn_set_conv_kernel": (c_int, [c_void_p, c_int]),
    "cnnue_synth_rn_weights": (c_int, [c_u64] + [P] * 14),
    "cnnue_synth_rn_planes": (c_int, [c_u64, c_i64, P]),
    "cnnue_splitmix64_next": (c_u64, [C.POINTER(c_u64)]),
    "cnnue_synth_positions": (c_int, [c_u64, c_i64, c_u32, c_u32, c_u32, P, P, C.POINTER(c_u32)]),
    "cnnue_synth_q_weights": (c_int, [c_u64, P, P, P, P, P, P, P, P]),
    "cnnue_synth_f_weights": (c_int, [c_u64, P, P, P, P, P, P, P, P]),
    "cnnue_synth_q_update": (c_int, [c_u64, c_i64, P, P, P, P, C.POINTER(c_u32), P, P,
                                     C.POINTER(c_u32), P]),
}

_lib = None


class CnnueError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str = ""):
        self.status = status
        msg = f"{where}: {status_string(status)}"
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)


def lib() -> C.CDLL:
    """Loads libcnnue.so (once) and declares every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m chineseai_b200.build` "
            "(the evaluator has no CPU fallback)")
    handle = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


def status_string(status: int) -> str:
    return lib().cnnue_status_string(status).decode()


def last_error() -> str:
    return lib().cnnue_last_error().decode()


def check(status: int, where: str) -> None:
    if status != 0:
        raise CnnueError(status, where, last_error())
