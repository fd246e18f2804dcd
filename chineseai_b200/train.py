"""Data-parallel training step of the HalfKA network (host side over the C ABI).

`Trainer` holds the flat fp32 parameters, the Adam moments and the bf16
shadow of the FT on one GPU.  One `step` = the rank's forward + backward in
libcnnue (gather, pack, bucket stack, loss, atomic-free FT backward, bucketed
stack gradients), one sum all-reduce of the flat gradient over the process
group (NCCL over NVLink between GPUs), then Adam with the gradient divided by
the world size.  It takes the role of the reference trainer's batch step
(GpuTrainer::train_batch_single / compute_batch_grads,
src/az/train_gpu_candle.rs:147-219) for this network.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from ._lib import check, lib
from .quantized import _stream_ptr, as_device
from .synth import Positions

N_FEATURES = 11340
COLS = 1024
BUCKETS = 16

# flat layout: name -> shape, in order
LAYOUT = (
    ("ft", (N_FEATURES, COLS)),
    ("ft_bias", (COLS,)),
    ("w1", (BUCKETS, 16, COLS)),
    ("b1", (BUCKETS, 16)),
    ("w2", (BUCKETS, 32, 16)),
    ("b2", (BUCKETS, 32)),
    ("w3", (BUCKETS, 32)),
    ("b3", (BUCKETS,)),
)
SHADOW = N_FEATURES * COLS + COLS


def param_count() -> int:
    return int(lib().cnnue_t_param_count())


def split(flat):
    """Views of a flat parameter (or gradient) array by name."""
    out, o = {}, 0
    for name, shape in LAYOUT:
        n = int(np.prod(shape))
        out[name] = flat[o:o + n].reshape(shape)
        o += n
    return out


def init_params(seed: int = 3) -> np.ndarray:
    """Seeded initial parameters (fp32, flat layout).  Chosen so that FT
    activations and hidden units sit mostly inside the clipped-ReLU range."""
    rng = np.random.default_rng(seed)
    flat = np.empty(param_count(), np.float32)
    p = split(flat)
    p["ft"][:] = rng.normal(0.0, 0.05, p["ft"].shape)
    p["ft_bias"][:] = 0.25
    p["w1"][:] = rng.normal(0.0, 0.05, p["w1"].shape)
    p["b1"][:] = 0.1
    p["w2"][:] = rng.normal(0.0, 0.2, p["w2"].shape)
    p["b2"][:] = 0.1
    p["w3"][:] = rng.normal(0.0, 10.0, p["w3"].shape)
    p["b3"][:] = 0.0
    return flat


def targets(n: int, seed: int = 4) -> np.ndarray:
    return np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32)


@dataclass
class AdamConfig:
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8


def allreduce_sum_(grads: torch.Tensor, group=None, guard=None, step: int = 0) -> int:
    """Sums `grads` in place over the default (or given) process group and
    returns the world size (1 without torch.distributed).  With a
    dist_guard.StepGuard the peers' heartbeats for `step` are checked first
    and the collective is bounded (RankFailure instead of a hang)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return 1
    if guard is not None:
        guard.all_reduce(grads, step)
    else:
        dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=group)
    return dist.get_world_size(group)


class Trainer:
    def __init__(self, params: np.ndarray, device: int = 0, adam: AdamConfig = AdamConfig(), group=None,
                 guard=None):
        self.device = torch.device("cuda", device)
        self.adam = adam
        self.group = group
        self.guard = guard  # optional dist_guard.StepGuard for the exchange
        n = param_count()
        if params.shape != (n,):
            raise ValueError(f"expected {n} parameters, got {params.shape}")
        self.params = torch.from_numpy(np.ascontiguousarray(params, np.float32)).to(self.device)
        self.m = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.v = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.grads = torch.empty(n, dtype=torch.float32, device=self.device)
        self.shadow = torch.empty(SHADOW, dtype=torch.int16, device=self.device)
        self.loss = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.step_count = 0
        self._ws: Optional[torch.Tensor] = None
        check(lib().cnnue_t_make_shadow(self.params.data_ptr(), self.shadow.data_ptr(),
                                        _stream_ptr(None)), "cnnue_t_make_shadow")

    def workspace(self, n_positions: int, n_indices: int) -> torch.Tensor:
        need = int(lib().cnnue_t_workspace_bytes(n_positions, n_indices))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward_backward(self, idx: torch.Tensor, n_idx: int, off: torch.Tensor, n: int,
                         target: torch.Tensor, stream=None) -> None:
        ws = self.workspace(n, n_idx)
        check(lib().cnnue_t_forward_backward(self.params.data_ptr(), self.shadow.data_ptr(), idx.data_ptr(),
                                             n_idx, off.data_ptr(), n, target.data_ptr(),
                                             self.grads.data_ptr(), self.loss.data_ptr(), ws.data_ptr(),
                                             ws.numel(), _stream_ptr(stream)), "cnnue_t_forward_backward")

    def status(self, stream=None) -> int:
        st = C.c_int(0)
        check(lib().cnnue_read_status(self._ws.data_ptr(), _stream_ptr(stream), C.byref(st)), "cnnue_read_status")
        return st.value

    def apply_adam(self, grad_scale: float, stream=None) -> None:
        self.step_count += 1
        a = self.adam
        check(lib().cnnue_t_adam(self.params.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                                 self.grads.data_ptr(), self.shadow.data_ptr(), grad_scale, a.lr, a.beta1,
                                 a.beta2, a.eps, self.step_count, _stream_ptr(stream)), "cnnue_t_adam")

    def step(self, idx: torch.Tensor, n_idx: int, off: torch.Tensor, n: int, target: torch.Tensor) -> None:
        """One data-parallel step (asynchronous on the current stream)."""
        self.forward_backward(idx, n_idx, off, n, target)
        world = allreduce_sum_(self.grads, self.group, self.guard, self.step_count)
        self.apply_adam(1.0 / world)

    def step_positions(self, pos: Positions, target: np.ndarray) -> float:
        """Convenience: host batch -> one step; returns this rank's loss."""
        idx = as_device(pos.indices, self.device)
        off = as_device(pos.offsets, self.device)
        t = torch.from_numpy(np.ascontiguousarray(target, np.float32)).to(self.device)
        self.step(idx, len(pos.indices), off, pos.n, t)
        check(self.status(), "training step (kernel status)")
        return float(self.loss.item())
