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


OFF_W1 = N_FEATURES * COLS + COLS  # first stack parameter (the FT weights and bias come first)


class Trainer:
    """One rank of the HalfKA training step.

    With a process group of more than one rank the stack gradients (and a
    status flag) are all-reduced on a side stream while the FT gradient is
    still being reduced.  The FT gradient is then exchanged one of two ways:

    * shard=True (the default without a guard): one reduce-scatter leaves
      each rank the summed gradient of its 1/world of the FT parameters,
      Adam updates that shard (and the stack on every rank), and one
      all-gather of the bf16 shadow the forward reads rebuilds the whole
      table on every rank: 3/4 of an all-reduce's bytes and 1/world of the
      FT Adam.  The fp32 FT parameters of other ranks' shards are then stale
      on this rank; gather_state() all-gathers them (and the summed
      gradient) when the full fp32 state is needed (tests, checkpoints);
    * shard=False: `ft_chunks` row ranges, each all-reduced as soon as its
      rows are final, then Adam over everything on every rank.

    Adam waits for every exchange and is skipped on every rank when any
    rank's batch had bad input."""

    def __init__(self, params: np.ndarray, device: int = 0, adam: AdamConfig = AdamConfig(), group=None,
                 guard=None, ft_chunks: int = 1, shard: Optional[bool] = None):
        self.device = torch.device("cuda", device)
        self.adam = adam
        self.group = group
        self.guard = guard  # optional dist_guard.StepGuard for the exchange
        self.ft_chunks = ft_chunks
        self.shard = guard is None if shard is None else shard
        if self.shard and guard is not None:
            raise ValueError("the sharded exchange runs without a StepGuard; use shard=False with a guard")
        n = param_count()
        if params.shape != (n,):
            raise ValueError(f"expected {n} parameters, got {params.shape}")
        self.params = torch.from_numpy(np.ascontiguousarray(params, np.float32)).to(self.device)
        self.m = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.v = torch.zeros(n, dtype=torch.float32, device=self.device)
        # the gradient, then the status flag (reduced with the stack gradients)
        self._gbuf = torch.zeros(n + 64, dtype=torch.float32, device=self.device)
        self.grads = self._gbuf[:n]
        self.flag = self._gbuf[n:n + 1]
        self._side = None
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

    def apply_adam(self, grad_scale: float, stream=None, skip: Optional[torch.Tensor] = None) -> None:
        self.step_count += 1
        a = self.adam
        check(lib().cnnue_t_adam(self.params.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                                 self.grads.data_ptr(), self.shadow.data_ptr(), grad_scale, a.lr, a.beta1,
                                 a.beta2, a.eps, self.step_count, skip.data_ptr() if skip is not None else None,
                                 _stream_ptr(stream)), "cnnue_t_adam")

    def world(self) -> int:
        import torch.distributed as dist
        if not (dist.is_available() and dist.is_initialized()):
            return 1
        return dist.get_world_size(self.group)

    def step(self, idx: torch.Tensor, n_idx: int, off: torch.Tensor, n: int, target: torch.Tensor) -> None:
        """One data-parallel step (asynchronous on the current stream)."""
        if self.world() == 1:
            self.forward_backward(idx, n_idx, off, n, target)
            self.apply_adam(1.0)
            return
        self._step_overlapped(idx, n_idx, off, n, target)

    def _all_reduce(self, t: torch.Tensor, tag: int):
        """Sum all-reduce issued on the side stream (after its event waits);
        returns the work to wait on, or None when the guard ran it to
        completion."""
        import torch.distributed as dist
        if self.guard is not None:
            self.guard.all_reduce(t, 8 * self.step_count + tag)
            return None
        return dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group, async_op=True)

    def _shard_range(self):
        """(begin, end) of this rank's FT shard in flat parameter indices, or
        None when the FT does not split evenly (the all-reduce path runs)."""
        import torch.distributed as dist
        w = self.world()
        if OFF_W1 % w:
            return None
        size = OFF_W1 // w
        r = dist.get_rank(self.group)
        return r * size, (r + 1) * size

    def gather_state(self) -> None:
        """Sharded exchange: all-gathers the fp32 FT parameters and the summed
        FT gradient of every shard, so self.params and self.grads hold the
        whole state (as after an all-reduce step) on every rank."""
        import torch.distributed as dist
        sr = self._shard_range() if self.shard and self.world() > 1 else None
        if sr is None:
            return
        b, e = sr
        dist.all_gather_into_tensor(self.params[:OFF_W1], self.params[b:e], group=self.group)
        dist.all_gather_into_tensor(self.grads[:OFF_W1], self.grads[b:e], group=self.group)

    def _step_overlapped(self, idx, n_idx, off, n, target) -> None:
        ws = self.workspace(n, n_idx)
        s = torch.cuda.current_stream(self.device)
        sp = s.cuda_stream
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        L = lib()
        check(L.cnnue_t_forward_backward_begin(self.params.data_ptr(), self.shadow.data_ptr(), idx.data_ptr(), n_idx,
                                               off.data_ptr(), n, target.data_ptr(), self.grads.data_ptr(),
                                               ws.data_ptr(), ws.numel(), sp), "cnnue_t_forward_backward_begin")
        check(L.cnnue_t_finish(n, n_idx, self.loss.data_ptr(), ws.data_ptr(), ws.numel(), self.flag.data_ptr(), sp),
              "cnnue_t_finish")
        works = []

        def exchange(t, tag):
            ev = torch.cuda.Event()
            ev.record(s)
            with torch.cuda.stream(self._side):
                self._side.wait_event(ev)
                works.append(self._all_reduce(t, tag))

        exchange(self._gbuf[OFF_W1:param_count() + 1], 0)  # stack gradients + the status flag
        sr = self._shard_range() if self.shard else None
        if sr is not None:
            self._exchange_sharded(n, n_idx, ws, s, works, sr)
            return
        rows = N_FEATURES + 1
        bounds = [rows * k // self.ft_chunks for k in range(self.ft_chunks + 1)]
        for k in range(self.ft_chunks):
            rb, re = bounds[k], bounds[k + 1]
            check(L.cnnue_t_ft_grad_rows(n, n_idx, self.grads.data_ptr(), ws.data_ptr(), ws.numel(), rb, re, sp),
                  "cnnue_t_ft_grad_rows")
            exchange(self.grads[rb * COLS: re * COLS], 1 + k)
        for w in works:
            if w is not None:
                w.wait()  # the current stream waits for the collective
        ev = torch.cuda.Event()
        ev.record(self._side)
        s.wait_event(ev)
        self.apply_adam(1.0 / self.world(), skip=self.flag)

    def _exchange_sharded(self, n, n_idx, ws, s, works, sr) -> None:
        """FT gradient: one in-place reduce-scatter on the side stream; Adam
        on this rank's FT shard and on the stack; the shard's bf16 shadow
        all-gathered in place."""
        import torch.distributed as dist
        L = lib()
        sp = s.cuda_stream
        check(L.cnnue_t_ft_grad_rows(n, n_idx, self.grads.data_ptr(), ws.data_ptr(), ws.numel(), 0, N_FEATURES + 1,
                                     sp), "cnnue_t_ft_grad_rows")
        b, e = sr
        ev = torch.cuda.Event()
        ev.record(s)
        with torch.cuda.stream(self._side):
            self._side.wait_event(ev)
            works.append(dist.reduce_scatter_tensor(self.grads[b:e], self.grads[:OFF_W1], op=dist.ReduceOp.SUM,
                                                    group=self.group, async_op=True))
        for w in works:
            w.wait()  # the current stream waits for the collectives
        ev = torch.cuda.Event()
        ev.record(self._side)
        s.wait_event(ev)
        self.step_count += 1
        a = self.adam
        scale = 1.0 / self.world()
        for lo, hi in ((b, e), (OFF_W1, param_count())):
            check(L.cnnue_t_adam_range(self.params.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                                       self.grads.data_ptr(), self.shadow.data_ptr(), lo, hi, scale, a.lr, a.beta1,
                                       a.beta2, a.eps, self.step_count, self.flag.data_ptr(), sp),
                  "cnnue_t_adam_range")
        shadow = self.shadow.view(torch.bfloat16)
        dist.all_gather_into_tensor(shadow[:OFF_W1], shadow[b:e], group=self.group)

    def step_positions(self, pos: Positions, target: np.ndarray) -> float:
        """Convenience: host batch -> one step; returns this rank's loss."""
        idx = as_device(pos.indices, self.device)
        off = as_device(pos.offsets, self.device)
        t = torch.from_numpy(np.ascontiguousarray(target, np.float32)).to(self.device)
        self.step(idx, len(pos.indices), off, pos.n, t)
        check(self.status(), "training step (kernel status)")
        if self.world() > 1 and float(self.flag.item()) != 0.0:
            from ._lib import CnnueError
            raise CnnueError(2, "training step", "a rank's batch had bad input; no rank applied Adam")
        return float(self.loss.item())
