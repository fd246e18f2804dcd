"""The AZ-NNUE policy-head training ops (over the C ABI), with autograd.

`fused_policy`, `sparse_policy` and `tactical_policy` take the roles of the
reference's Candle custom ops of the same names (src/az/fused_policy.rs:
159-171, src/az/fused_sparse_policy.rs:56-62): same argument shapes, same
shape errors, backward passes through FusedPolicyGrad / SparsePolicyGrad's
arithmetic without atomics (deterministic, run to run and across batch
splits of the same items).  Item packing: `pack_policy_item` /
`padding_item` (src/az/fused_policy.rs:142-157).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import check, lib
from .quantized import _stream_ptr

TABLE_LEN = 182886
CONTEXT = 48
SPARSE_TERMS = 7
TACTICAL_TERMS = 2


def padding_item() -> int:
    return 0


def pack_policy_item(move_index: int, from_: int, to: int, captured: int, move_valid: bool,
                     capture_valid: bool) -> int:
    """move | from << 12 | to << 23 | captured << 34 | move_valid << 45 |
    capture_valid << 46 | policy_valid << 47, as a signed 64-bit value."""
    v = (move_index | from_ << 12 | to << 23 | captured << 34 | int(move_valid) << 45
         | int(capture_valid) << 46 | 1 << 47)
    return v


def _read_word(word: torch.Tensor) -> int:
    st = C.c_int(0)
    check(lib().cnnue_read_status(word.data_ptr(), _stream_ptr(None), C.byref(st)), "cnnue_read_status")
    return st.value


def _status_word(status, device):
    """(word the kernels OR into, whether to read it here).  A caller-owned
    int32 `status` tensor collects the bits of several ops without a host
    synchronisation; it is then the caller's to check."""
    if status is None:
        return torch.zeros(64, dtype=torch.int32, device=device), True
    return status, False


def _finish_ws(ws: torch.Tensor, status, where: str) -> None:
    """A backward op's workspace status: checked now, or ORed into `status`."""
    if status is None:
        check(_read_word(ws), where)
    else:
        status[:1].bitwise_or_(ws[:4].view(torch.int32))


def _contig(x: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if x.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {x.dtype}")
    return x.contiguous()


def fused_policy_forward(tables, context, items, status=None) -> torch.Tensor:
    batch, moves = items.shape
    out = torch.empty((batch, moves), dtype=torch.float32, device=tables.device)
    word, own = _status_word(status, tables.device)
    check(lib().cnnue_policy_fused_fwd(tables.data_ptr(), context.data_ptr(), items.data_ptr(), batch, moves,
                                       out.data_ptr(), word.data_ptr(), _stream_ptr(None)),
          "cnnue_policy_fused_fwd")
    if own:
        check(_read_word(word), "cnnue_policy_fused_fwd (kernel status)")
    return out


def fused_policy_backward(tables, context, items, grad_out, status=None):
    """-> (grad_tables [182886], grad_context [B, 48])."""
    batch, moves = items.shape
    gt = torch.empty(TABLE_LEN, dtype=torch.float32, device=tables.device)
    gc = torch.empty((batch, CONTEXT), dtype=torch.float32, device=tables.device)
    nbytes = int(lib().cnnue_policy_fused_bwd_workspace_bytes(batch, moves))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=tables.device)
    check(lib().cnnue_policy_fused_bwd(tables.data_ptr(), context.data_ptr(), items.data_ptr(),
                                       grad_out.data_ptr(), batch, moves, gt.data_ptr(), gc.data_ptr(),
                                       ws.data_ptr(), nbytes, _stream_ptr(None)), "cnnue_policy_fused_bwd")
    _finish_ws(ws, status, "cnnue_policy_fused_bwd (kernel status)")
    return gt, gc


class _FusedPolicy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tables, context, items, status):
        ctx.save_for_backward(tables, context, items)
        ctx.status = status
        return fused_policy_forward(tables, context, items, status)

    @staticmethod
    def backward(ctx, grad_out):
        tables, context, items = ctx.saved_tensors
        gt, gc = fused_policy_backward(tables, context, items, grad_out.contiguous().float(), ctx.status)
        return gt, gc, None, None


def fused_policy(tables: torch.Tensor, context: torch.Tensor, items: torch.Tensor, status=None) -> torch.Tensor:
    """tables f32 [182886], context f32 [B, 48], items i64 [B, M] -> logits f32 [B, M].
    `status` (int32 device tensor): collect kernel status bits there instead
    of checking them (and synchronising) in every call."""
    if tables.dim() != 1 or context.dim() != 2 or items.dim() != 2 or tables.shape[0] != TABLE_LEN \
            or context.shape[1] != CONTEXT or items.shape[0] != context.shape[0]:
        raise ValueError(f"fused policy shape mismatch: tables={tuple(tables.shape)}, "
                         f"context={tuple(context.shape)}, items={tuple(items.shape)}")
    return _FusedPolicy.apply(_contig(tables, torch.float32, "tables"), _contig(context, torch.float32, "context"),
                              _contig(items, torch.int64, "items"), status)


def table_forward(table, indices, status=None) -> torch.Tensor:
    terms = indices.shape[-1]
    outputs = indices.numel() // terms
    out = torch.empty(indices.shape[:-1], dtype=torch.float32, device=table.device)
    word, own = _status_word(status, table.device)
    check(lib().cnnue_policy_table_fwd(table.data_ptr(), table.numel(), indices.data_ptr(), outputs, terms,
                                       out.data_ptr(), word.data_ptr(), _stream_ptr(None)),
          "cnnue_policy_table_fwd")
    if own:
        check(_read_word(word), "cnnue_policy_table_fwd (kernel status)")
    return out


def table_backward(indices, grad_out, table_len: int, status=None) -> torch.Tensor:
    terms = indices.shape[-1]
    outputs = indices.numel() // terms
    grad = torch.empty(table_len, dtype=torch.float32, device=indices.device)
    nbytes = int(lib().cnnue_policy_table_bwd_workspace_bytes(outputs, terms))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=indices.device)
    check(lib().cnnue_policy_table_bwd(indices.data_ptr(), grad_out.data_ptr(), outputs, terms, table_len,
                                       grad.data_ptr(), ws.data_ptr(), nbytes, _stream_ptr(None)),
          "cnnue_policy_table_bwd")
    _finish_ws(ws, status, "cnnue_policy_table_bwd (kernel status)")
    return grad


class _TablePolicy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, table, indices, status):
        ctx.save_for_backward(indices)
        ctx.table_len = table.numel()
        ctx.status = status
        return table_forward(table, indices, status)

    @staticmethod
    def backward(ctx, grad_out):
        (indices,) = ctx.saved_tensors
        return table_backward(indices, grad_out.contiguous().float(), ctx.table_len, ctx.status), None, None


def _table_policy(table: torch.Tensor, indices: torch.Tensor, expected_terms: int, status=None) -> torch.Tensor:
    if table.dim() != 1 or indices.dim() != 3:
        raise ValueError(f"sparse policy expects a 1-D table and [B, M, terms] indices, got "
                         f"{tuple(table.shape)} and {tuple(indices.shape)}")
    terms = indices.shape[2]
    if terms != expected_terms:
        raise ValueError(f"sparse policy expects {expected_terms} indices per move, got {terms}")
    return _TablePolicy.apply(_contig(table, torch.float32, "table"), _contig(indices, torch.int64, "indices"),
                              status)


def sparse_policy(tables: torch.Tensor, indices: torch.Tensor, status=None) -> torch.Tensor:
    """tables f32 [L], indices i64 [B, M, 7] -> f32 [B, M] (seven lookups summed)."""
    return _table_policy(tables, indices, SPARSE_TERMS, status)


def tactical_policy(tables: torch.Tensor, indices: torch.Tensor, status=None) -> torch.Tensor:
    """tables f32 [L], indices i64 [B, M, 2] -> f32 [B, M] (two lookups summed)."""
    return _table_policy(tables, indices, TACTICAL_TERMS, status)
