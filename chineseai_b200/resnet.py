"""Host-side API of the AlphaZero policy/value ResNet (over the C ABI).

`ResNetWeights` holds the fp32 host weights in PyTorch layouts (synthetic,
seeded: `ResNetWeights.synthetic(seed)`); `ResNetModel` uploads them to one GPU
(conv weights as bf16 tiles for the tensor cores) and evaluates leaf batches
of bf16 input planes [B][15][10][9] into policy probabilities [B][2086],
optional logits and values [B].  The network takes the evaluator's place for
MCTS leaf batches (AzNnue::evaluate_with_scratch_output, src/az.rs:1562-1604;
src/az/alphazero.rs:388-521); every computation runs in libcnnue's kernels.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields
from typing import Optional

import numpy as np

from ._lib import check, lib

PLANES, CHANNELS, BLOCKS, MOVES, SQUARES = 15, 128, 10, 2086, 90


class RnWeightsC(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "stem_w", "stem_b", "block_w", "block_b", "policy_conv_w", "policy_conv_b", "policy_fc_w", "policy_fc_b",
        "value_conv_w", "value_conv_b", "value_fc1_w", "value_fc1_b", "value_fc2_w", "value_fc2_b")]


@dataclass
class ResNetWeights:
    stem_w: np.ndarray         # [128][15][3][3]
    stem_b: np.ndarray         # [128]
    block_w: np.ndarray        # [10][2][128][128][3][3]
    block_b: np.ndarray        # [10][2][128]
    policy_conv_w: np.ndarray  # [2][128]
    policy_conv_b: np.ndarray  # [2]
    policy_fc_w: np.ndarray    # [2086][180]
    policy_fc_b: np.ndarray    # [2086]
    value_conv_w: np.ndarray   # [128]
    value_conv_b: np.ndarray   # [1]
    value_fc1_w: np.ndarray    # [256][90]
    value_fc1_b: np.ndarray    # [256]
    value_fc2_w: np.ndarray    # [256]
    value_fc2_b: np.ndarray    # [1]

    SHAPES = {"stem_w": (128, 15, 3, 3), "stem_b": (128,), "block_w": (10, 2, 128, 128, 3, 3),
              "block_b": (10, 2, 128), "policy_conv_w": (2, 128), "policy_conv_b": (2,),
              "policy_fc_w": (2086, 180), "policy_fc_b": (2086,), "value_conv_w": (128,), "value_conv_b": (1,),
              "value_fc1_w": (256, 90), "value_fc1_b": (256,), "value_fc2_w": (256,), "value_fc2_b": (1,)}

    @classmethod
    def synthetic(cls, seed: int = 5) -> "ResNetWeights":
        arrays = {k: np.zeros(v, np.float32) for k, v in cls.SHAPES.items()}
        check(lib().cnnue_synth_rn_weights(seed, *[arrays[f.name].ctypes.data for f in fields(cls)]),
              "cnnue_synth_rn_weights")
        return cls(**arrays)

    def arrays(self):
        return [np.ascontiguousarray(getattr(self, f.name), np.float32) for f in fields(self)]


def synthetic_planes(batch: int, seed: int = 6) -> np.ndarray:
    """bf16 bits uint16 [B][15][10][9]."""
    planes = np.zeros((batch, PLANES, 10, 9), np.uint16)
    check(lib().cnnue_synth_rn_planes(seed, batch, planes.ctypes.data if batch else None), "cnnue_synth_rn_planes")
    return planes


def bf16_to_float(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


class ResNetModel:
    def __init__(self, weights: ResNetWeights, device: int = 0):
        import torch
        self._torch = torch
        self.device = torch.device("cuda", device)
        self._keep = weights.arrays()
        cw = RnWeightsC(*[a.ctypes.data for a in self._keep])
        h = C.c_void_p()
        check(lib().cnnue_rn_model_create(C.byref(cw), device, C.byref(h)), "cnnue_rn_model_create")
        self._h = h
        self._ws = None

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cnnue_rn_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    CONV_KERNELS = {"tile": 0, "persistent": 1, "halo": 2}

    def set_conv_kernel(self, kind: str) -> None:
        """Chooses the trunk conv kernel: "halo" (default; padded 8-board
        layout, one halo tile per channel half), "persistent" or "tile"
        (square-major layout, one TMA box per tap).  All compute the same
        convolution; only the summation order inside the tensor cores may
        differ."""
        check(lib().cnnue_rn_set_conv_kernel(self._h, self.CONV_KERNELS[kind]), "cnnue_rn_set_conv_kernel")

    def workspace(self, batch: int):
        need = int(lib().cnnue_rn_workspace_bytes(batch))
        if self._ws is None or self._ws.numel() < need:
            self._ws = self._torch.empty(need, dtype=self._torch.uint8, device=self.device)
        return self._ws

    def read_status(self, stream=None) -> int:
        st = C.c_int(0)
        s = stream if stream is not None else self._torch.cuda.current_stream(self.device)
        check(lib().cnnue_read_status(self._ws.data_ptr(), s.cuda_stream, C.byref(st)), "cnnue_read_status")
        return st.value

    def forward(self, planes, with_logits: bool = False, stream=None):
        """planes: device int16/uint16 tensor of bf16 bits [B][15][10][9].
        Returns (probs [B][2086], logits or None, value [B])."""
        torch = self._torch
        batch = planes.shape[0]
        probs = torch.empty((batch, MOVES), dtype=torch.float32, device=self.device)
        logits = torch.empty((batch, MOVES), dtype=torch.float32, device=self.device) if with_logits else None
        value = torch.empty(batch, dtype=torch.float32, device=self.device)
        ws = self.workspace(batch)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(lib().cnnue_rn_forward(self._h, planes.data_ptr(), batch, probs.data_ptr(),
                                     logits.data_ptr() if logits is not None else None, value.data_ptr(),
                                     ws.data_ptr(), ws.numel(), s.cuda_stream), "cnnue_rn_forward")
        return probs, logits, value
