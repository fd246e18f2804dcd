"""Host-side API of the quantised HalfKA evaluator (over the C ABI).

`QuantizedNnue` is the device-resident evaluator: it owns the weights on one
GPU and evaluates batches given as CSR feature lists.  It takes the role of the
reference's `AzNnue` evaluator object (src/az.rs:861-901; construction
src/az.rs:1339-1529; batch evaluation src/az.rs:1562-1736) for this network.

Device buffers are torch CUDA tensors (torch is used for device memory and
streams only); every computation runs in libcnnue's kernels.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np
import torch

from ._lib import QWeights, check, lib
from .synth import Positions, QuantizedWeights, UpdateBatch, quantized_weights


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def as_device(a: np.ndarray, device: torch.device) -> torch.Tensor:
    """Copies a numpy array to the device as raw bytes of the same width
    (uint16 -> int16, uint32 -> int32 views; only the pointer matters)."""
    view = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32}.get(a.dtype)
    host = np.ascontiguousarray(a).view(view) if view is not None else np.ascontiguousarray(a)
    return torch.from_numpy(host).to(device)


class QuantizedNnue:
    """Quantised HalfKA NNUE (int16 FT 11340x1024, 16 int8 bucket stacks)."""

    def __init__(self, weights: QuantizedWeights, device: int = 0):
        self.device = torch.device("cuda", device)
        self.weights = weights
        arrays = weights.arrays()
        cw = QWeights(*[a.ctypes.data for a in arrays])
        handle = C.c_void_p()
        check(lib().cnnue_q_model_create(C.byref(cw), device, C.byref(handle)), "cnnue_q_model_create")
        self._h = handle
        self._ws: Optional[torch.Tensor] = None

    @classmethod
    def random(cls, seed: int = 2, device: int = 0) -> "QuantizedNnue":
        return cls(quantized_weights(seed), device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_q_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    # ---- workspace ----------------------------------------------------------
    @staticmethod
    def workspace_bytes(n_positions: int) -> int:
        return int(lib().cnnue_q_workspace_bytes(n_positions))

    def workspace(self, n_positions: int) -> torch.Tensor:
        need = self.workspace_bytes(n_positions)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def read_status(self, workspace: torch.Tensor, stream=None) -> int:
        st = C.c_int(0)
        check(lib().cnnue_read_status(workspace.data_ptr(), _stream_ptr(stream), C.byref(st)),
              "cnnue_read_status")
        return st.value

    # ---- evaluation ---------------------------------------------------------
    def forward(self, indices: torch.Tensor, offsets: torch.Tensor, n_positions: int,
                out: Optional[torch.Tensor] = None, acc_out: Optional[torch.Tensor] = None,
                workspace: Optional[torch.Tensor] = None, stream=None,
                check_status: bool = True) -> torch.Tensor:
        """Scores (int32 [n]) of device-resident positions.  `indices` holds
        uint16 values (any 2-byte dtype), `offsets` uint32 values (any 4-byte
        dtype), both contiguous on this model's device."""
        if out is None:
            out = torch.empty(n_positions, dtype=torch.int32, device=self.device)
        ws = workspace if workspace is not None else self.workspace(n_positions)
        sp = _stream_ptr(stream)
        if acc_out is None:
            st = lib().cnnue_q_forward(self._h, indices.data_ptr(), indices.numel(), offsets.data_ptr(),
                                       n_positions, out.data_ptr(), ws.data_ptr(), ws.numel(), sp)
        else:
            st = lib().cnnue_q_forward_acc(self._h, indices.data_ptr(), indices.numel(),
                                           offsets.data_ptr(), n_positions, out.data_ptr(),
                                           acc_out.data_ptr(), ws.data_ptr(), ws.numel(), sp)
        check(st, "cnnue_q_forward")
        if check_status and n_positions > 0:
            check(self.read_status(ws, stream), "cnnue_q_forward (kernel status)")
        return out

    def forward_positions(self, pos: Positions, with_acc: bool = False):
        """Convenience: host Positions -> (scores np.int32[n], acc np.int16[n,2,1024] | None)."""
        idx = as_device(pos.indices, self.device)
        off = as_device(pos.offsets, self.device)
        acc = None
        if with_acc:
            acc = torch.empty((pos.n, 2, 1024), dtype=torch.int16, device=self.device)
        scores = self.forward(idx, off, pos.n, acc_out=acc)
        torch.cuda.synchronize(self.device)
        return scores.cpu().numpy(), (acc.cpu().numpy() if acc is not None else None)

    def forward_host(self, indices: np.ndarray, offsets: np.ndarray, out: Optional[np.ndarray] = None,
                     stream=None) -> np.ndarray:
        """End-to-end call with host buffers (pinned or pageable numpy arrays)."""
        n = (len(offsets) - 1) // 2
        if out is None:
            out = np.empty(n, dtype=np.int32)
        check(lib().cnnue_q_forward_host(self._h, indices.ctypes.data, len(indices), offsets.ctypes.data,
                                         n, out.ctypes.data, _stream_ptr(stream)),
              "cnnue_q_forward_host")
        return out

    def pipeline(self, max_positions: int, max_indices: int) -> "HostPipeline":
        """A pipelined host-buffer evaluator (one per thread) over this model."""
        return HostPipeline(self, max_positions, max_indices)

    def update(self, batch: UpdateBatch, stream=None):
        """Incremental update + stack: returns (child acc np.int16[n,2,1024], scores np.int32[n])."""
        d = self.device
        parent = as_device(batch.parent, d)
        flags = as_device(batch.flags, d)
        rem = as_device(batch.rem if len(batch.rem) else np.zeros(1, np.uint16), d)
        add = as_device(batch.add if len(batch.add) else np.zeros(1, np.uint16), d)
        ro = as_device(batch.rem_offsets, d)
        ao = as_device(batch.add_offsets, d)
        c0 = as_device(batch.count0, d)
        n = batch.n
        child = torch.empty((n, 2, 1024), dtype=torch.int16, device=d)
        scores = torch.empty(n, dtype=torch.int32, device=d)
        ws = self.workspace(n)
        check(lib().cnnue_q_update(self._h, parent.data_ptr(), flags.data_ptr(), rem.data_ptr(),
                                   len(batch.rem), ro.data_ptr(), add.data_ptr(), len(batch.add),
                                   ao.data_ptr(), c0.data_ptr(), n, child.data_ptr(), scores.data_ptr(),
                                   ws.data_ptr(), ws.numel(), _stream_ptr(stream)), "cnnue_q_update")
        if n > 0:
            check(self.read_status(ws, stream), "cnnue_q_update (kernel status)")
        torch.cuda.synchronize(d)
        return child.cpu().numpy(), scores.cpu().numpy()


class HostPipeline:
    """Two-slot pipelined evaluation of host batches (cnnue_q_ctx_*): `submit`
    enqueues a batch and returns a ticket at once, `wait` returns its status
    once the scores are in the caller's output array.  Up to two batches are
    in flight, so one batch's host-to-device copies overlap the previous
    batch's kernels.  Use pinned numpy arrays (e.g. from
    torch.empty(..., pin_memory=True).numpy()) for asynchronous copies; the
    arrays of a batch must stay untouched until its wait returns."""

    def __init__(self, model: QuantizedNnue, max_positions: int, max_indices: int):
        self.model = model
        h = C.c_void_p()
        check(lib().cnnue_q_ctx_create(model.handle, max_positions, max_indices, C.byref(h)), "cnnue_q_ctx_create")
        self._h = h
        self._keep = {}

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_q_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def next_stream(self) -> int:
        s = C.c_void_p()
        check(lib().cnnue_q_ctx_next_stream(self._h, C.byref(s)), "cnnue_q_ctx_next_stream")
        return s.value or 0

    def submit(self, indices: np.ndarray, offsets: np.ndarray, out: np.ndarray) -> int:
        n = (len(offsets) - 1) // 2
        t = C.c_uint64(0)
        check(lib().cnnue_q_forward_host_async(self._h, indices.ctypes.data, len(indices), offsets.ctypes.data, n,
                                               out.ctypes.data, C.byref(t)), "cnnue_q_forward_host_async")
        self._keep[t.value] = (indices, offsets, out)
        return t.value

    def wait(self, ticket: int) -> int:
        st = C.c_int(0)
        check(lib().cnnue_q_ctx_wait(self._h, ticket, C.byref(st)), "cnnue_q_ctx_wait")
        self._keep.pop(ticket, None)
        return st.value
