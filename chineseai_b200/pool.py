"""The AZ-NNUE trunk feature pool and the plain table pool (over the C ABI).

`feature_pool` / `feature_pool_backward` take the roles of the reference's
Candle ops feature_pool and FeaturePoolGrad (src/az/fused_feature_pool.rs:
134-148, 214-223); `sparse_pool` / `sparse_pool_backward` those of
sparse_pool / SparsePoolGrad (:150-163, :276-282).  Items use the reference's
packing: feature | us_bucket << 11 | them_bucket << 15, 0xffffffff = padding.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import check, lib
from .quantized import _stream_ptr

POOL_ROWS = 1545
PADDING_ITEM = 0xFFFFFFFF


def pack_feature(feature: int, us_bucket: int, them_bucket: int) -> int:
    return feature | (us_bucket << 11) | (them_bucket << 15)


def _read_word(word: torch.Tensor, stream=None) -> int:
    st = C.c_int(0)
    check(lib().cnnue_read_status(word.data_ptr(), _stream_ptr(stream), C.byref(st)), "cnnue_read_status")
    return st.value


def _status_word(status, device):
    if status is None:
        return torch.zeros(64, dtype=torch.int32, device=device), True
    return status, False


def _finish_ws(ws: torch.Tensor, status, stream, where: str) -> None:
    if status is None:
        check(_read_word(ws, stream), where)
    else:
        status[:1].bitwise_or_(ws[:4].view(torch.int32))


class _FeaturePool(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tables, items, status):
        ctx.save_for_backward(items)
        ctx.status = status
        return _feature_pool_fwd(tables, items, None, status)

    @staticmethod
    def backward(ctx, grad_out):
        (items,) = ctx.saved_tensors
        return feature_pool_backward(items, grad_out.contiguous(), status=ctx.status), None, None


class _SparsePool(torch.autograd.Function):
    @staticmethod
    def forward(ctx, table, items, status):
        ctx.save_for_backward(items)
        ctx.rows = table.shape[0]
        ctx.status = status
        return _sparse_pool_fwd(table, items, None, status)

    @staticmethod
    def backward(ctx, grad_out):
        (items,) = ctx.saved_tensors
        return sparse_pool_backward(items, grad_out.contiguous(), ctx.rows, status=ctx.status), None, None


def feature_pool(tables: torch.Tensor, items: torch.Tensor, stream=None, status=None) -> torch.Tensor:
    """tables f32 [1545, H] (cuda), items [B, I] 4-byte (cuda) -> f32 [B, H].
    Differentiable in `tables` (backward: feature_pool_backward) when called
    on the current stream.  `status` (int32 device tensor): collect kernel
    status bits there instead of checking them (and synchronising) here."""
    if stream is None and torch.is_grad_enabled() and tables.requires_grad:
        return _FeaturePool.apply(tables, items, status)
    return _feature_pool_fwd(tables, items, stream, status)


def _feature_pool_fwd(tables: torch.Tensor, items: torch.Tensor, stream=None, status=None) -> torch.Tensor:
    rows, hidden = tables.shape
    if rows != POOL_ROWS:
        raise ValueError(f"feature pool row mismatch: got {rows}, expected {POOL_ROWS}")
    batch, item_count = items.shape
    out = torch.empty((batch, hidden), dtype=torch.float32, device=tables.device)
    word, own = _status_word(status, tables.device)
    check(lib().cnnue_feature_pool_fwd(tables.data_ptr(), items.data_ptr(), batch, item_count, hidden,
                                       out.data_ptr(), word.data_ptr(), _stream_ptr(stream)),
          "cnnue_feature_pool_fwd")
    if own:
        check(_read_word(word, stream), "cnnue_feature_pool_fwd (kernel status)")
    return out


def feature_pool_backward(items: torch.Tensor, grad_out: torch.Tensor, stream=None, status=None) -> torch.Tensor:
    """Gradient of feature_pool w.r.t. the tables: f32 [1545, H]."""
    batch, item_count = items.shape
    hidden = grad_out.shape[1]
    grad = torch.empty((POOL_ROWS, hidden), dtype=torch.float32, device=grad_out.device)
    nbytes = int(lib().cnnue_feature_pool_bwd_workspace_bytes(batch, item_count, hidden))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=grad_out.device)
    check(lib().cnnue_feature_pool_bwd(items.data_ptr(), grad_out.data_ptr(), batch, item_count, hidden,
                                       grad.data_ptr(), ws.data_ptr(), nbytes, _stream_ptr(stream)),
          "cnnue_feature_pool_bwd")
    _finish_ws(ws, status, stream, "cnnue_feature_pool_bwd (kernel status)")
    return grad


def sparse_pool(table: torch.Tensor, items: torch.Tensor, stream=None, status=None) -> torch.Tensor:
    """table f32 [R, H], items [B, I] 4-byte row indices (0xffffffff padding)
    -> f32 [B, H]; differentiable in `table` like feature_pool."""
    if stream is None and torch.is_grad_enabled() and table.requires_grad:
        return _SparsePool.apply(table, items, status)
    return _sparse_pool_fwd(table, items, stream, status)


def _sparse_pool_fwd(table: torch.Tensor, items: torch.Tensor, stream=None, status=None) -> torch.Tensor:
    rows, hidden = table.shape
    batch, item_count = items.shape
    out = torch.empty((batch, hidden), dtype=torch.float32, device=table.device)
    word, own = _status_word(status, table.device)
    check(lib().cnnue_sparse_pool_fwd(table.data_ptr(), rows, items.data_ptr(), batch, item_count, hidden,
                                      out.data_ptr(), word.data_ptr(), _stream_ptr(stream)),
          "cnnue_sparse_pool_fwd")
    if own:
        check(_read_word(word, stream), "cnnue_sparse_pool_fwd (kernel status)")
    return out


def sparse_pool_backward(items: torch.Tensor, grad_out: torch.Tensor, rows: int, stream=None,
                         status=None) -> torch.Tensor:
    batch, item_count = items.shape
    hidden = grad_out.shape[1]
    grad = torch.empty((rows, hidden), dtype=torch.float32, device=grad_out.device)
    nbytes = int(lib().cnnue_sparse_pool_bwd_workspace_bytes(rows, batch, item_count, hidden))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=grad_out.device)
    check(lib().cnnue_sparse_pool_bwd(items.data_ptr(), grad_out.data_ptr(), rows, batch, item_count, hidden,
                                      grad.data_ptr(), ws.data_ptr(), nbytes, _stream_ptr(stream)),
          "cnnue_sparse_pool_bwd")
    _finish_ws(ws, status, stream, "cnnue_sparse_pool_bwd (kernel status)")
    return grad
