"""Host-side API of the fp32 HalfKA evaluator (over the C ABI)."""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np
import torch

from ._lib import FWeights, check, lib
from .quantized import _stream_ptr, as_device
from .synth import FloatWeights, Positions, float_weights


class FloatNnue:
    """fp32 HalfKA NNUE (FT 11340x256 per perspective, 8 bucket stacks 512->16->32->1)."""

    def __init__(self, weights: FloatWeights, device: int = 0):
        self.device = torch.device("cuda", device)
        self.weights = weights
        cw = FWeights(*[a.ctypes.data for a in weights.arrays()])
        handle = C.c_void_p()
        check(lib().cnnue_f_model_create(C.byref(cw), device, C.byref(handle)), "cnnue_f_model_create")
        self._h = handle
        self._ws: Optional[torch.Tensor] = None

    @classmethod
    def random(cls, seed: int = 2, device: int = 0) -> "FloatNnue":
        return cls(float_weights(seed), device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_f_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, indices: torch.Tensor, offsets: torch.Tensor, n_positions: int,
                out: Optional[torch.Tensor] = None, stream=None, check_status: bool = True) -> torch.Tensor:
        if out is None:
            out = torch.empty(n_positions, dtype=torch.float32, device=self.device)
        need = int(lib().cnnue_f_workspace_bytes(n_positions))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        ws = self._ws
        check(lib().cnnue_f_forward(self._h, indices.data_ptr(), indices.numel(), offsets.data_ptr(),
                                    n_positions, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                    _stream_ptr(stream)), "cnnue_f_forward")
        if check_status and n_positions > 0:
            st = C.c_int(0)
            check(lib().cnnue_read_status(ws.data_ptr(), _stream_ptr(stream), C.byref(st)), "cnnue_read_status")
            check(st.value, "cnnue_f_forward (kernel status)")
        return out

    def forward_positions(self, pos: Positions) -> np.ndarray:
        idx = as_device(pos.indices if len(pos.indices) else np.zeros(1, np.uint16), self.device)
        off = as_device(pos.offsets, self.device)
        out = self.forward(idx[: len(pos.indices)] if len(pos.indices) else idx, off, pos.n)
        torch.cuda.synchronize(self.device)
        return out.cpu().numpy()
