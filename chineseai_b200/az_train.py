"""AZ-NNUE training: samples, the native batch packer, and the training step.

`pack_batch` takes the role of PackedBatch::from_indices
(src/az/dataloader.rs:113-336) through the C ABI (cnnue_az_pack_batch,
multi-threaded C++); `AzTrainer` that of GpuTrainer
(src/az/train_gpu_candle.rs:15-160): AzCandleModel::forward
(src/az/candle_model.rs:46-147) composed from this package's CUDA ops
(feature_pool, sparse_pool, fused_policy, sparse_policy, tactical_policy)
and dense cuBLAS matmuls, the loss of compute_batch_loss
(src/az/train_gpu_candle.rs:221-305), autograd, and the AdamW step of
candle-nn (lr, betas 0.9 / 0.999, eps 1e-8, weight decay 1e-4) as one CUDA
kernel over a flat parameter buffer.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields
from typing import Optional

import numpy as np

from . import az
from ._lib import check, lib

DENSE_MOVES = 2086
RULE_CONTEXT = 7
POLICY_MASK_VALUE = -1.0e9
SPARSE_TABLE = 2396815
SPARSE_FACTOR = 199458
TACTICAL = 934976


@dataclass
class Samples:
    """Training samples in CSR form (the AzTrainingSample fields the packer
    reads): canonical side-to-move features per sample, move indices with
    their policy targets, WDL / value targets, rule context, loss weights, ply."""
    features: np.ndarray         # u16 [total]
    feature_offsets: np.ndarray  # u32 [n + 1]
    move_indices: np.ndarray     # u16 [total moves]
    policy: np.ndarray           # f32 [total moves]
    move_offsets: np.ndarray     # u32 [n + 1]
    value_wdl: np.ndarray        # f32 [n, 3]
    value: np.ndarray            # f32 [n]
    rule_context: np.ndarray     # f32 [n, 7]
    policy_weight: np.ndarray    # f32 [n]
    value_weight: np.ndarray     # f32 [n]
    ply: np.ndarray              # u32 [n]

    @property
    def n(self) -> int:
        return len(self.feature_offsets) - 1


def random_samples(n: int, seed: int, max_moves: int = 40) -> Samples:
    """Synthetic samples of the self-play format: random boards (az.random_boards),
    a random side to move, its canonical features in board-scan order, up to
    `max_moves` pseudo moves in the dense space with gamma-distributed visit
    targets, random WDL / value / rule context / weights / ply.  A few samples
    carry the cases the packer must handle: features >= 1260, move indices
    >= 2086, moves whose source square holds no own piece, negative targets
    and weights, all-zero WDL, out-of-range values."""
    rng = np.random.default_rng(seed)
    boards = az.random_boards(n, seed ^ 0x5EED)
    _, s2d = az.dense_moves()
    feats, foff, moves, pol, moff = [], [0], [], [], [0]
    for i in range(n):
        side = int(rng.integers(0, 2))
        f = (az.features(boards[i], side) & 0x7FF).astype(np.uint16)
        if rng.random() < 0.05:
            f = np.append(f, np.uint16(1260 + rng.integers(0, 100)))
        feats.append(f)
        foff.append(foff[-1] + len(f))
        mv = az.pseudo_moves(boards[i], side, rng, int(rng.integers(1, max_moves + 1)))
        cf = mv[:, 0].astype(np.int64) if side == 0 else 89 - mv[:, 0].astype(np.int64)
        ct = mv[:, 1].astype(np.int64) if side == 0 else 89 - mv[:, 1].astype(np.int64)
        dense = s2d[cf * 90 + ct].astype(np.uint16)
        if rng.random() < 0.1:
            dense = np.append(dense, np.uint16(rng.integers(0, DENSE_MOVES)))  # any move, maybe no own piece
        if rng.random() < 0.05:
            dense = np.append(dense, np.uint16(DENSE_MOVES + rng.integers(0, 50)))  # outside the move space
        p = rng.gamma(0.5, 1.0, size=len(dense)).astype(np.float32)
        if rng.random() < 0.05:
            p[:] = 0.0
        if rng.random() < 0.05 and len(p):
            p[0] = -0.5
        moves.append(dense)
        pol.append(p)
        moff.append(moff[-1] + len(dense))
    wdl = rng.dirichlet([1.0, 1.0, 1.0], size=n).astype(np.float32)
    wdl[rng.random(n) < 0.03] = 0.0
    return Samples(
        features=np.concatenate(feats).astype(np.uint16) if feats else np.zeros(0, np.uint16),
        feature_offsets=np.array(foff, np.uint32),
        move_indices=np.concatenate(moves).astype(np.uint16) if moves else np.zeros(0, np.uint16),
        policy=np.concatenate(pol).astype(np.float32) if pol else np.zeros(0, np.float32),
        move_offsets=np.array(moff, np.uint32),
        value_wdl=wdl,
        value=rng.uniform(-1.2, 1.2, size=n).astype(np.float32),
        rule_context=rng.standard_normal((n, RULE_CONTEXT)).astype(np.float32),
        policy_weight=rng.uniform(-0.1, 1.5, size=n).astype(np.float32),
        value_weight=rng.uniform(-0.1, 1.5, size=n).astype(np.float32),
        ply=rng.integers(0, 200, size=n).astype(np.uint32),
    )


class _CSamples(C.Structure):
    _fields_ = [("n", C.c_int64)] + [(name, C.c_void_p) for name in (
        "features", "feature_offsets", "move_indices", "policy", "move_offsets", "value_wdl", "value",
        "rule_context", "policy_weight", "value_weight", "ply")]


@dataclass
class PackedBatch:
    """PackedBatch (src/az/dataloader.rs:92-111) as numpy arrays.  A compact
    batch carries policy_signature / king_buckets instead of the sparse,
    tactical and mask arrays (None), which the GPU rebuilds."""
    feature_items: np.ndarray           # u32 [B, F]
    value_threat_indices: np.ndarray    # u32 [B, T]
    policy_items: np.ndarray            # i64 [B, M]
    policy_sparse_indices: Optional[np.ndarray]    # i64 [B, M, 7]
    policy_tactical_indices: Optional[np.ndarray]  # i64 [B, M, 2]
    policy_targets: np.ndarray          # f32 [B, M]
    policy_mask: Optional[np.ndarray]   # f32 [B, M]
    value_wdl: np.ndarray               # f32 [B, 3]
    values: np.ndarray                  # f32 [B]
    rule_context: np.ndarray            # f32 [B, 7]
    policy_weights: np.ndarray          # f32 [B]
    value_weights: np.ndarray           # f32 [B]
    value_phase_masks: np.ndarray       # f32 [B, 3]
    policy_signature: Optional[np.ndarray] = None  # u8 [B, M] (compact)
    king_buckets: Optional[np.ndarray] = None      # u8 [B] us | them << 4 (compact)

    @property
    def batch_size(self) -> int:
        return self.values.shape[0]

    @property
    def compact(self) -> bool:
        return self.policy_sparse_indices is None


_PACKED_FIELDS = [f.name for f in fields(PackedBatch)]


class _CAztBatch(C.Structure):
    """cnnue_azt_batch: the packed batch's device arrays (full form)."""
    _fields_ = [(n, C.c_int64) for n in ("batch", "features", "moves", "threats")] + \
        [(n, C.c_void_p) for n in (
            "feature_items", "value_threat_indices", "policy_items", "policy_sparse_indices",
            "policy_tactical_indices", "policy_targets", "policy_mask", "value_wdl", "values", "rule_context",
            "policy_weights", "value_weights", "value_phase_masks")]


NATIVE_HIDDEN = (32, 64, 128, 256, 512)  # hidden sizes of the native step (cnnue_azt_step)


class _CAztOptim(C.Structure):
    """cnnue_azt_optim: AdamW inside the native step."""
    _fields_ = [(n, C.c_void_p) for n in ("params", "m", "v", "state")]


class _CPacked(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("batch", "max_features", "max_policy_moves", "max_value_threats")] + \
        [(name, C.c_void_p) for name in _PACKED_FIELDS]


def _samples_struct(s: Samples, keep: list) -> _CSamples:
    arrays = [np.ascontiguousarray(a, dt) for a, dt in (
        (s.features, np.uint16), (s.feature_offsets, np.uint32), (s.move_indices, np.uint16),
        (s.policy, np.float32), (s.move_offsets, np.uint32), (s.value_wdl, np.float32), (s.value, np.float32),
        (s.rule_context, np.float32), (s.policy_weight, np.float32), (s.value_weight, np.float32),
        (s.ply, np.uint32))]
    arrays = [a if a.size else np.zeros(1, a.dtype) for a in arrays]
    keep.extend(arrays)
    return _CSamples(s.n, *[a.ctypes.data for a in arrays])


def pack_batch(samples: Samples, rows: Optional[np.ndarray] = None, n_threads: int = 0,
               caps=(96, 160, 256), fixed: bool = False, compact: bool = False) -> PackedBatch:
    """Packs samples[rows] (all samples when rows is None) with the native
    packer.  fixed=True: the arrays take the `caps` widths whatever the batch
    needs (CnnueError if it needs more), for a trainer with a captured step.
    compact=True: per-move tactical signatures and per-row king buckets
    instead of the 7 + 2 int64 lookup indices and the mask (the trainer
    rebuilds those on the GPU: about a fifth of the bytes to send)."""
    keep: list = []
    cs = _samples_struct(samples, keep)
    if rows is None:
        batch, rptr = samples.n, None
    else:
        r = np.ascontiguousarray(rows, np.int64)
        keep.append(r)
        batch, rptr = len(r), (r.ctypes.data if len(r) else None)
    while True:
        F, M, T = caps
        b = max(batch, 1)
        bufs = {
            "feature_items": np.empty((b, F), np.uint32), "value_threat_indices": np.empty((b, T), np.uint32),
            "policy_items": np.empty((b, M), np.int64), "policy_sparse_indices": np.empty((b, M, 7), np.int64),
            "policy_tactical_indices": np.empty((b, M, 2), np.int64), "policy_targets": np.empty((b, M), np.float32),
            "policy_mask": np.empty((b, M), np.float32), "value_wdl": np.empty((b, 3), np.float32),
            "values": np.empty(b, np.float32), "rule_context": np.empty((b, RULE_CONTEXT), np.float32),
            "policy_weights": np.empty(b, np.float32), "value_weights": np.empty(b, np.float32),
            "value_phase_masks": np.empty((b, 3), np.float32),
            "policy_signature": np.empty((b, M), np.uint8), "king_buckets": np.empty(b, np.uint8)}
        if compact:
            for k in ("policy_sparse_indices", "policy_tactical_indices", "policy_mask"):
                bufs[k] = None
        else:
            bufs["policy_signature"] = bufs["king_buckets"] = None
        out = _CPacked(0, 0, 0, 0, *[None if bufs[k] is None else bufs[k].ctypes.data for k in _PACKED_FIELDS])
        st = lib().cnnue_az_pack_batch(C.byref(cs), rptr, batch, F, M, T, int(fixed), C.byref(out), n_threads)
        need = (out.max_features, out.max_policy_moves, out.max_value_threats)
        if st == 5 and not fixed and any(n > c for n, c in zip(need, caps)):  # CNNUE_ERR_WORKSPACE: grow, retry
            caps = tuple(max(n, c) for n, c in zip(need, caps))
            continue
        check(st, "cnnue_az_pack_batch")
        break
    F, M, T = need

    def cut(a, width, extra=()):
        if a is None:
            return None
        flat = a.reshape(-1)[: batch * width * int(np.prod(extra or (1,)))]
        return flat.reshape((batch, width) + tuple(extra))

    return PackedBatch(
        feature_items=cut(bufs["feature_items"], F), value_threat_indices=cut(bufs["value_threat_indices"], T),
        policy_items=cut(bufs["policy_items"], M), policy_sparse_indices=cut(bufs["policy_sparse_indices"], M, (7,)),
        policy_tactical_indices=cut(bufs["policy_tactical_indices"], M, (2,)),
        policy_targets=cut(bufs["policy_targets"], M), policy_mask=cut(bufs["policy_mask"], M),
        value_wdl=bufs["value_wdl"][:batch], values=bufs["values"][:batch],
        rule_context=bufs["rule_context"][:batch], policy_weights=bufs["policy_weights"][:batch],
        value_weights=bufs["value_weights"][:batch], value_phase_masks=bufs["value_phase_masks"][:batch],
        policy_signature=cut(bufs["policy_signature"], M),
        king_buckets=None if bufs["king_buckets"] is None else bufs["king_buckets"][:batch])


# ---- the training step --------------------------------------------------------
def mean_allreduce_(grad, group=None) -> int:
    """grad <- the mean of grad over the ranks of `group` (sum all-reduce, then
    1 / world); returns the world size.  With equal shares of the batch per
    rank this is the gradient of the whole batch's mean loss."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=group)
    grad.mul_(1.0 / world)
    return world


# Tail of the gradient buffer: 30 metrics, then 4 status-bit indicators.
_TAIL = 64
_N_METRICS = 30
_NATIVE_OUT = _N_METRICS + 5  # the native step's metrics: 30 statistics, 4 status bits (0/1), the word


def exchange_with_status_(buf, n_grad: int, tail_at: int, metrics, word, group=None, read: bool = True,
                          guard=None, step: int = 0):
    """The data-parallel exchange of one training step, in one sum
    all-reduce over `group`: buf[:n_grad] holds this rank's gradient and
    becomes the ranks' mean; buf[tail_at:] receives this rank's metrics
    (summed over the ranks: the whole batch's sums) and its kernel status
    word as four 0/1 bit indicators (a sum above zero means some rank set the
    bit, so every rank reads the same OR).  Returns (metrics sums, status
    word) as host values when `read`, else None (no host synchronisation).
    With a dist_guard.StepGuard the peers' heartbeats for `step` are checked
    before the collective and the collective is bounded (RankFailure)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    tail = buf[tail_at: tail_at + _N_METRICS + 4]
    tail[:_N_METRICS].copy_(metrics[:_N_METRICS])
    w = torch.as_tensor(word).to(device=buf.device, dtype=torch.int32).reshape(())
    tail[_N_METRICS:].copy_(torch.stack([((w >> b) & 1).float() for b in range(4)]))
    if guard is not None:
        guard.all_reduce(buf, step)
    else:
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    buf[:n_grad].mul_(1.0 / world)
    if not read:
        return None
    m = tail.cpu().numpy()
    return m[:_N_METRICS].copy(), sum(1 << b for b in range(4) if m[_N_METRICS + b] > 0)


def _raise_status(word: int, where: str) -> None:
    """The kernels' status bits as cnnue_read_status maps them."""
    if word == 0:
        return
    from ._lib import CnnueError
    code = 3 if word & 2 else (2 if word & 1 else (9 if word & 4 else 10))
    raise CnnueError(code, where, f"kernel status word 0x{word:x}")


# Leaves of the flat parameter buffer: (name, first tensor, last tensor, shape).
# Tensors 0-4 form the [1545, H] feature table of feature_pool, 19-20 the
# sparse policy table, and the tactical table (last) carries one constant
# zero after it (the Tensor::zeros(1) of candle_model.rs:133-139).
_LEAVES = [
    ("feature_tables", 0, 4, lambda h: (1545, h)),
    ("rule_context_hidden", 5, 5, lambda h: (RULE_CONTEXT, h)),
    ("hidden_bias", 6, 6, lambda h: (h,)),
    ("value_head_hidden", 7, 7, lambda h: (96, h)),
    ("value_head_bias", 8, 8, lambda h: (96,)),
    ("value_head_output", 9, 9, lambda h: (3, 96)),
    ("value_threat_embedding", 10, 10, lambda h: (57702, 64)),
    ("value_threat_output", 11, 11, lambda h: (3, 128)),
    ("policy_threat_context", 12, 12, lambda h: (16, 128)),
    ("policy_move_bias", 13, 13, lambda h: (DENSE_MOVES,)),
    ("policy_consequence_output", 14, 14, lambda h: (32,)),
    ("policy_context_hidden", 15, 15, lambda h: (16, h)),
    ("policy_move_context", 16, 16, lambda h: (DENSE_MOVES, 16)),
    ("policy_accumulator_hidden", 17, 17, lambda h: (32, h)),
    ("policy_accumulator_move", 18, 18, lambda h: (DENSE_MOVES, 32)),
    ("sparse_tables", 19, 20, lambda h: (SPARSE_TABLE + SPARSE_FACTOR,)),
    ("tactical_table", 21, 21, lambda h: (TACTICAL + 1,)),
]
_ALIGN = 64  # floats: every leaf starts on a 256-byte boundary


@dataclass
class TrainStats:
    """AzTrainStats of one batch (src/az/train_gpu_candle.rs:271-300): sums
    over the batch (loss = weighted CE sum, not yet divided by the batch)."""
    loss: float
    value_loss: float
    policy_ce: float
    value_pred_sum: float
    value_pred_sq_sum: float
    value_target_sum: float
    value_target_sq_sum: float
    value_pred_target_sum: float
    value_error_sq_sum: float
    samples: int
    phase: np.ndarray  # [3][7]: samples, pred, pred^2, target, target^2, pred*target, error^2 sums


class AzTrainer:
    """GpuTrainer (src/az/train_gpu_candle.rs:15-160) on one CUDA device.

    native (default for hidden 32/64/128/256/512): the step is the native
    kernel sequence cnnue_azt_step (forward, both losses, all gradients);
    native=False: torch autograd around this package's CUDA ops.

    graph=True captures the whole step (forward, loss, backward, AdamW) in a
    CUDA graph once a batch shape repeats (batches packed with fixed=True all
    share one shape), and replays it; the first step of each new shape runs
    eagerly.  The AdamW step counter and learning rate live in device memory
    (cnnue_adamw_device), so replays advance them.

    group: a torch.distributed process group (NCCL) for data parallelism:
    every rank steps on its own equal share of the batch, the flat gradient is
    sum-all-reduced once and scaled by 1 / world (the gradient of the whole
    batch's mean loss), and every rank applies the same AdamW update.  The
    native step without a guard keeps that exchange on the device (metrics
    and status bits written into the all-reduced gradient tail, AdamW
    skipped on the device when any rank set a status bit), so a captured
    graph holds the whole data-parallel step; call close() before
    destroy_process_group.  With a guard (or native=False) the exchange and
    AdamW run after the step, from the host.  Either way the step's
    statistics (TrainStats) are the whole batch's (sums over every rank's
    share, samples = the global batch), and a kernel status raised on any
    rank skips AdamW and raises on every rank."""

    def __init__(self, weights: "az.AzWeights", lr: float = 1e-3, device: int = 0, weight_decay: float = 1e-4,
                 beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8, graph: bool = False, group=None,
                 guard=None, native: Optional[bool] = None):
        import torch
        self.torch = torch
        if native is None:
            native = weights.hidden in NATIVE_HIDDEN
        if native and weights.hidden not in NATIVE_HIDDEN:
            raise ValueError(f"the native step supports hidden sizes {NATIVE_HIDDEN}, got {weights.hidden}")
        self.native = native
        self._engine = None
        self.use_graph = graph
        self.group = group
        self.guard = guard  # optional dist_guard.StepGuard for the exchange
        self.world = 1
        if group is not None:
            import torch.distributed as dist
            self.world = dist.get_world_size(group)
        self._graph = None
        self._graph_key = None
        self._last_key = None
        self.hidden = h = weights.hidden
        self.device = torch.device("cuda", device)
        self.lr, self.beta1, self.beta2, self.eps, self.weight_decay = lr, beta1, beta2, eps, weight_decay
        self.step_count = 0
        sizes = [az.tensor_info(i, h)[1] for i in range(az.N_TENSORS)]
        starts = np.concatenate([[0], np.cumsum(sizes)])
        layout, pos = [], 0
        for name, first, last, shape in _LEAVES:
            n = int(starts[last + 1] - starts[first]) + (1 if name == "tactical_table" else 0)
            layout.append((name, first, last, shape(h), pos, n))
            pos = pos + n if name == "tactical_table" else (pos + n + _ALIGN - 1) // _ALIGN * _ALIGN
        self.n_params = pos - 1  # AdamW covers everything but the tactical table's constant zero
        host = np.zeros(pos, np.float32)
        for name, first, last, shape, off, n in layout:
            host[off:off + int(starts[last + 1] - starts[first])] = np.concatenate(
                [weights.tensor(i).reshape(-1) for i in range(first, last + 1)])
        self.flat = torch.from_numpy(host).to(self.device)
        # the gradient, then (data parallel) a tail that carries the step's
        # metrics and status bits through the same all-reduce
        self._tail_at = (pos + _ALIGN - 1) // _ALIGN * _ALIGN
        self.grad = torch.zeros(self._tail_at + _TAIL, dtype=torch.float32, device=self.device)
        self.m = torch.zeros(self.n_params, dtype=torch.float32, device=self.device)
        self.v = torch.zeros_like(self.m)
        self._layout = layout
        self.params = {}
        for name, first, last, shape, off, n in layout:
            p = torch.nn.Parameter(self.flat[off:off + n].view(shape))
            p.grad = self.grad[off:off + n].view(shape)
            self.params[name] = p
        self._wdl_q = torch.tensor([1.0, 0.0, -1.0], device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._pinned = None
        self._arena = None
        # cnnue_adamw_state: lr, beta1, beta2, eps, weight_decay (f64), step (i64), 12 floats
        state = np.zeros(12, np.float64)
        state[:5] = [lr, beta1, beta2, eps, weight_decay]
        self.adam_state = torch.from_numpy(state.view(np.uint8).copy()).to(self.device)
        # native step: leaf offsets of the flat buffers, metrics, workspaces by batch shape
        self._leaf_offsets = np.array([off for _, _, _, _, off, _ in layout], np.int64)
        self._metrics = torch.zeros(_NATIVE_OUT, dtype=torch.float32, device=self.device)
        self._ws = {}
        if self.native:
            e = C.c_void_p()
            check(lib().cnnue_azt_create(device, C.byref(e)), "cnnue_azt_create")
            self._engine = e

    def close(self) -> None:
        """Releases the captured step (before destroy_process_group when it
        holds the NCCL exchange) and the native step's engine."""
        self._graph = None
        if self._engine is not None:
            lib().cnnue_azt_destroy(self._engine)
            self._engine = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_learning_rate(self, lr: float) -> None:
        """GpuTrainer::set_learning_rate (src/az/train_gpu_candle.rs:134-136)."""
        self.lr = lr
        self.adam_state[:8].copy_(self.torch.from_numpy(np.array([lr], np.float64).view(np.uint8)))

    # -- data ---------------------------------------------------------------
    def to_device(self, b: PackedBatch) -> dict:
        """BatchTensors::from_packed (src/az/candle_model.rs:173-233): the
        batch's arrays staged in one pinned host buffer and sent in one copy;
        the device tensors are views of one device buffer (valid until the
        next call)."""
        torch = self.torch
        arrays, offsets, total = [], [], 0
        for f in fields(PackedBatch):
            if getattr(b, f.name) is None:
                continue
            a = np.ascontiguousarray(getattr(b, f.name))
            if a.dtype == np.uint32:
                a = a.view(np.int32)
            arrays.append((f.name, a))
            offsets.append(total)
            total += (a.nbytes + 255) // 256 * 256
        if self._pinned is None or self._pinned.numel() < total:
            self._pinned = torch.empty(total, dtype=torch.uint8, pin_memory=True)
            self._arena = torch.empty(total, dtype=torch.uint8, device=self.device)
        host = self._pinned.numpy()
        for (name, a), off in zip(arrays, offsets):
            host[off:off + a.nbytes] = a.reshape(-1).view(np.uint8)
        self._arena[:total].copy_(self._pinned[:total], non_blocking=True)
        self._last_h2d = total
        dt = {np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64, np.dtype(np.float32): torch.float32,
              np.dtype(np.uint8): torch.uint8}
        return {name: self._arena[off:off + a.nbytes].view(dt[a.dtype]).view(a.shape)
                for (name, a), off in zip(arrays, offsets)}

    def expand(self, bt: dict) -> dict:
        """A compact batch's sparse / tactical indices and mask, rebuilt on the
        GPU (cnnue_az_expand_policy_indices); full batches pass through."""
        if "policy_signature" not in bt:
            return bt
        torch = self.torch
        items = bt["policy_items"]
        B, M = items.shape
        sparse = torch.empty((B, M, 7), dtype=torch.int64, device=self.device)
        tactical = torch.empty((B, M, 2), dtype=torch.int64, device=self.device)
        mask = torch.empty((B, M), dtype=torch.float32, device=self.device)
        check(lib().cnnue_az_expand_policy_indices(items.data_ptr(), bt["policy_signature"].data_ptr(),
                                                   bt["king_buckets"].data_ptr(), B, M, sparse.data_ptr(),
                                                   tactical.data_ptr(), mask.data_ptr(),
                                                   torch.cuda.current_stream(self.device).cuda_stream),
              "cnnue_az_expand_policy_indices")
        out = dict(bt)
        out.update(policy_sparse_indices=sparse, policy_tactical_indices=tactical, policy_mask=mask)
        return out

    @property
    def h2d_bytes(self) -> int:
        """Bytes of the last batch's host-to-device copy."""
        return 0 if self._pinned is None else int(self._last_h2d)

    # -- model ----------------------------------------------------------------
    def forward(self, bt: dict):
        """AzCandleModel::forward (src/az/candle_model.rs:46-147) ->
        (value_logits [B, 3], policy_logits [B, M])."""
        from . import policy as pol
        from . import pool
        torch = self.torch
        P = self.params
        h = self.hidden
        ft = P["feature_tables"]
        st = self.status
        board_pre = pool.feature_pool(ft, bt["feature_items"], status=st) + P["hidden_bias"]
        accumulator_context = board_pre @ P["policy_accumulator_hidden"].t()
        rule_pre = bt["rule_context"] @ P["rule_context_hidden"]
        sparse_hidden = torch.relu(board_pre + rule_pre)
        rms = torch.sqrt((sparse_hidden * sparse_hidden).mean(1, keepdim=True) + 1.0e-6)
        hidden = sparse_hidden / rms
        value_head = torch.relu(hidden @ P["value_head_hidden"].t() + P["value_head_bias"])
        value_logits = value_head @ P["value_head_output"].t()
        threat_acc = pool.sparse_pool(P["value_threat_embedding"], bt["value_threat_indices"], status=st)
        threat_act = threat_acc.clamp(0.0, 1.0)
        threat_pair = torch.cat([threat_act, threat_act * threat_act], 1)
        value_logits = value_logits + threat_pair @ P["value_threat_output"].t()
        input_hidden = ft[:1260]
        cs = min(32, h)
        psp = input_hidden[:, :cs]
        if cs < 32:
            psp = torch.cat([psp, psp.new_zeros(1260, 32 - cs)], 1)
        policy_context = hidden @ P["policy_context_hidden"].t() + threat_pair @ P["policy_threat_context"].t()
        policy_context = torch.cat([policy_context, accumulator_context], 1)
        accumulator_feature = input_hidden @ P["policy_accumulator_hidden"].t()
        tables = torch.cat([psp.reshape(-1), P["policy_consequence_output"], P["policy_move_bias"],
                            P["policy_move_context"].reshape(-1), accumulator_feature.reshape(-1),
                            P["policy_accumulator_move"].reshape(-1)])
        policy_logits = pol.fused_policy(tables, policy_context, bt["policy_items"], st)
        policy_logits = policy_logits + pol.sparse_policy(P["sparse_tables"], bt["policy_sparse_indices"], st)
        policy_logits = policy_logits + pol.tactical_policy(P["tactical_table"], bt["policy_tactical_indices"], st)
        return value_logits, policy_logits

    def loss(self, bt: dict, value_weight: float = 1.0, policy_weight: float = 1.0):
        """compute_batch_loss (src/az/train_gpu_candle.rs:221-305) -> (loss
        tensor = weighted CE sum / B, metrics tensor [30])."""
        torch = self.torch
        value_logits, policy_logits = self.forward(bt)
        value_log_probs = torch.log_softmax(value_logits, 1)
        value = (value_log_probs.exp() @ self._wdl_q)
        value_ce_ps = (bt["value_wdl"] * value_log_probs * -1.0).sum(1)
        log_policy = torch.log_softmax(policy_logits + bt["policy_mask"], 1)
        policy_ce_ps = (bt["policy_targets"] * log_policy * -1.0).sum(1)
        weighted_value = (value_ce_ps * bt["value_weights"]).sum() * max(value_weight, 0.0)
        weighted_policy = (policy_ce_ps * bt["policy_weights"]).sum() * max(policy_weight, 0.0)
        loss_sum = weighted_value + weighted_policy
        batch = bt["values"].shape[0]
        loss = loss_sum / batch
        with torch.no_grad():
            target = bt["values"]
            err = value - target
            per = torch.stack([value, value * value, target, target * target, value * target, err * err], 1)
            phase = bt["value_phase_masks"].t() @ torch.cat([torch.ones_like(value)[:, None], per], 1)  # [3, 7]
            metrics = torch.cat([torch.stack([loss_sum, value_ce_ps.sum(), policy_ce_ps.sum()]), per.sum(0),
                                 phase.reshape(-1)])
        return loss, metrics

    def native_loss(self, bt: dict, value_weight: float = 1.0, policy_weight: float = 1.0, out=None,
                    adamw: bool = False):
        """The native step's forward, loss and backward (cnnue_azt_step) on a
        device batch: the 22 gradients land in self.grad (zeroed first);
        returns the metrics tensor [35] (`out`, default an own buffer): the
        30 statistics of compute_batch_loss, the status word's 4 bits as 0/1,
        the word as a float.  adamw=True also applies AdamW (single GPU): the
        table leaves' update runs while the dense gradients finish."""
        torch = self.torch
        bt = self.expand(bt)
        B, F = bt["feature_items"].shape
        M = bt["policy_items"].shape[1]
        T = bt["value_threat_indices"].shape[1]
        key = (B, F, M, T)
        ws = self._ws.get(key)
        if ws is None:
            nbytes = int(lib().cnnue_azt_workspace_bytes(self.hidden, B, F, M, T))
            if nbytes == 0:
                raise ValueError(f"native step: unsupported batch dims {key} at hidden {self.hidden}")
            ws = self._ws[key] = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        names = [f[0] for f in _CAztBatch._fields_[4:]]
        arrays = {n: bt["values" if n == "values" else n] for n in names}
        for n, a in arrays.items():
            if not a.is_contiguous():
                raise ValueError(f"native step: batch array {n} is not contiguous")
        batch = _CAztBatch(B, F, M, T, *[arrays[n].data_ptr() for n in names])
        out = self._metrics if out is None else out
        optim = _CAztOptim(self.flat.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                           self.adam_state.data_ptr()) if adamw else None
        check(lib().cnnue_azt_step(self._engine, self.flat.data_ptr(), self.grad.data_ptr(), self._tail_at,
                                   self._leaf_offsets.ctypes.data, self.hidden, C.byref(batch),
                                   float(value_weight), float(policy_weight), out.data_ptr(),
                                   self.status.data_ptr(), ws.data_ptr(), ws.numel(),
                                   C.byref(optim) if optim is not None else None,
                                   torch.cuda.current_stream(self.device).cuda_stream), "cnnue_azt_step")
        return out

    def _in_graph_exchange(self) -> bool:
        """Native data-parallel steps without a guard keep the whole exchange
        on the device: metrics and status bits in the gradient tail, one NCCL
        sum all-reduce, AdamW scaled by 1/world and skipped on the device when
        any rank set a status bit - so a captured step holds all of it."""
        return self.native and self.world > 1 and self.guard is None

    def _step_body(self, bt: dict, value_weight: float, policy_weight: float):
        if self._in_graph_exchange():
            import torch.distributed as dist
            out = self.grad[self._tail_at: self._tail_at + _NATIVE_OUT]
            self.native_loss(bt, value_weight, policy_weight, out)
            dist.all_reduce(self.grad, op=dist.ReduceOp.SUM, group=self.group)
            check(lib().cnnue_adamw_device_scaled(self.flat.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                                                  self.grad.data_ptr(), self.n_params, self.adam_state.data_ptr(),
                                                  1.0 / self.world, out[_N_METRICS:].data_ptr(), 4,
                                                  self.torch.cuda.current_stream(self.device).cuda_stream),
                  "cnnue_adamw_device_scaled")
            return out
        if self.native:
            return self.native_loss(bt, value_weight, policy_weight, adamw=self.world == 1)
        self.grad.zero_()
        self.status.zero_()
        loss, metrics = self.loss(self.expand(bt), value_weight, policy_weight)
        loss.backward()
        if self.world == 1:
            self._adamw()
        return self.torch.cat([metrics, self.status.float()])

    def _adamw(self) -> None:
        check(lib().cnnue_adamw_device(self.flat.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                                       self.grad.data_ptr(), self.n_params, self.adam_state.data_ptr(),
                                       self.torch.cuda.current_stream(self.device).cuda_stream),
              "cnnue_adamw_device")

    def _exchange(self, out, read: bool = True):
        """Data parallel: one NCCL sum all-reduce carries the gradient and
        every rank's metrics and status bits (exchange_with_status_); all
        ranks then take the same decision on AdamW."""
        r = exchange_with_status_(self.grad, self.n_params, self._tail_at, out, out[-1], self.group, read,
                                  self.guard, self.step_count)
        if r is None:
            return None
        return np.concatenate([r[0], [float(r[1])]])

    def step(self, batch: PackedBatch, value_weight: float = 1.0, policy_weight: float = 1.0) -> TrainStats:
        """One train_batch_single (src/az/train_gpu_candle.rs:145-160):
        forward, loss, backward, AdamW; one host synchronisation, at the end
        (metrics and the kernels' status word come back together).  A bad
        index in the batch raises CnnueError after the step."""
        torch = self.torch
        bt = self.to_device(batch)
        self.step_count += 1
        key = (tuple((k, tuple(v.shape)) for k, v in bt.items()), self._arena.data_ptr(), value_weight,
               policy_weight)
        if not self.use_graph:
            out = self._step_body(bt, value_weight, policy_weight)
        elif self._graph is not None and key == self._graph_key:
            self._graph.replay()
            out = self._graph_out
        elif key == self._last_key:  # the shape repeats: capture it, then replay this step
            self._graph = None
            g = torch.cuda.CUDAGraph()
            torch.cuda.synchronize(self.device)
            with torch.cuda.graph(g):
                self._graph_out = self._step_body(bt, value_weight, policy_weight)
            self._graph, self._graph_key = g, key
            g.replay()
            out = self._graph_out
        else:
            out = self._step_body(bt, value_weight, policy_weight)
        self._last_key = key
        samples = batch.batch_size
        if self._in_graph_exchange():
            t = out.cpu().numpy()  # summed over the ranks by the step's all-reduce
            word = sum(1 << b for b in range(4) if t[_N_METRICS + b] > 0)
            m = np.concatenate([t[:_N_METRICS], [float(word)]])
            samples *= self.world
        elif self.world > 1:
            m = self._exchange(out)
            samples *= self.world
            if int(m[-1]) == 0:  # every rank applies the step, or none does
                self._adamw()
        else:
            m = out.cpu().numpy()
        _raise_status(int(m[-1]), "AzTrainer.step")
        return TrainStats(*[float(x) for x in m[:9]], samples=samples, phase=m[9:30].reshape(3, 7))

    # -- weights ------------------------------------------------------------------
    def tensors(self) -> list:
        """The 22 weight tensors (host numpy copies) in the reference layout."""
        h = self.hidden
        host = self.flat.cpu().numpy()
        out = []
        for name, first, last, shape, off, n in self._layout:
            pos = off
            for i in range(first, last + 1):
                k = az.tensor_info(i, h)[1]
                out.append(host[pos:pos + k].reshape(az.tensor_shape(i, h)).copy())
                pos += k
        return out

    def copy_to(self, weights: "az.AzWeights") -> None:
        """copy_to_model (src/az/train_gpu_candle.rs:162-164); re-quantises."""
        for i, t in enumerate(self.tensors()):
            weights.tensor(i)[...] = t
        weights.quantize()

    def gradients(self) -> list:
        """The last step's gradients as 22 host arrays (reference layout)."""
        h = self.hidden
        host = self.grad.cpu().numpy()
        out = []
        for name, first, last, shape, off, n in self._layout:
            pos = off
            for i in range(first, last + 1):
                k = az.tensor_info(i, h)[1]
                out.append(host[pos:pos + k].reshape(az.tensor_shape(i, h)).copy())
                pos += k
        return out
