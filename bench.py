#!/usr/bin/env python
"""Benchmark of the quantised NNUE evaluation hot path on B200.

Workload (one step): the quantised HalfKA NNUE forward of a batch of 65,536
positions - per position and perspective 2-32 unique active features out of
11,340, int16 FT of 1024 columns with wraparound, pairwise clipped-ReLU pack
to 1024 uint8, 16 bucket int8 stacks 1024->16->32->1 - on synthetic inputs
(SplitMix64 seed 1 + rank for positions, seed 2 for weights).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0.  `value` is device-resident throughput (inputs in HBM,
L2 flushed between steps); `e2e` is the same metric through the pipelined
host-buffer C ABI (cnnue_q_forward_host_async: pinned H2D copy of every step's
indices/offsets and D2H of its scores inside the timed region, two steps in
flight).  `--impl reference` times the CPU evaluator (the
oracle restatement; the Rust reference cannot be built) on all host threads.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BATCH = 65536
METRIC = "NNUE evals/sec (int8/int16, batch 64K)"
UNIT = "evals/s"
WORKLOAD = ("quantized HalfKA NNUE forward: F=11340, int16 FT 11340x1024 shared by 2 perspectives "
            "(wraparound), 2-32 unique sorted active features per perspective, pairwise clipped-ReLU "
            "pack to 1024 u8, bucket=(n0-1)/2 of 16 int8 stacks 1024->16->32->1")
L2_FLUSH_BYTES = 256 << 20
HBM_FALLBACK_GBS = 6650.0
# Stack weights and FT bias, read once per batch (16 buckets).
STACK_BYTES = 16 * (16 * 1024 + 16 * 4 + 32 * 16 + 32 * 4 + 32 + 4) + 2048


def algorithmic_bytes(n_positions: int, n_indices: int) -> int:
    """Bytes one forward must move: every gathered FT row (2 KB) once per use,
    the uint16 indices, the uint32 offsets, the int32 scores, and the stack
    weights once per batch."""
    return n_indices * 2048 + n_indices * 2 + (2 * n_positions + 1) * 4 + n_positions * 4 + STACK_BYTES


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def committed_traffic():
    """DRAM bytes per forward (gather + stack kernels) from the committed ncu
    summary (profiles/q_forward_b65536.json) of a 65,536-position launch."""
    path = os.path.join(ROOT, "profiles", "q_forward_b65536.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return int(d["dram_bytes_per_launch_65536"])
    except Exception:
        return None


# ---------------------------------------------------------------------------
# reference arm: the CPU evaluator on all host threads
# ---------------------------------------------------------------------------
def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_cpu_model() -> str:
    """Host CPU: model name, sockets x cores per socket, logical CPUs, and
    whether the timed CPU path runs its AVX2 kernels."""
    model, cores, sockets = "unknown", None, set()
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name") and model == "unknown":
                model = line.split(":", 1)[1].strip()
            elif line.startswith("cpu cores") and cores is None:
                cores = int(line.split(":", 1)[1])
            elif line.startswith("physical id"):
                sockets.add(line.split(":", 1)[1].strip())
    except Exception:
        pass
    try:
        import oracle
        avx2 = bool(oracle.lib().oracle_q_has_avx2())
    except Exception:
        avx2 = False
    return (f"{model}, {max(len(sockets), 1)} socket(s) x {cores} cores, {os.cpu_count()} logical CPUs, "
            f"{'AVX2 kernels' if avx2 else 'scalar kernels'}")


def cpu_time_batches(w, pos, threads: int, min_seconds: float, min_reps: int):
    import oracle
    reps, t0 = 0, time.perf_counter()
    while True:
        st, _ = oracle.q_forward_mt(w, pos, threads)
        if st != 0:
            raise RuntimeError(f"oracle status {st}")
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= min_seconds:
            return reps, el


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from chineseai_b200 import synth
    threads = cpu_threads()
    w = synth.quantized_weights(2)
    pos = synth.positions(BATCH, 1)
    cpu_time_batches(w, pos, threads, 0.0, max(args.warmup, 1))
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        import oracle
        st, _ = oracle.q_forward_mt(w, pos, threads)
        times.append(time.perf_counter() - t0)
        assert st == 0
    ms = 1e3 * sum(times) / len(times)
    value = BATCH / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": BATCH, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"full {BATCH}-position batch per step, {threads} OpenMP threads, "
                                   f"CPU {cpu_cpu_model()}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import ctypes as C

    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    from chineseai_b200 import synth
    from chineseai_b200._lib import check, lib
    from chineseai_b200.quantized import QuantizedNnue, as_device

    L = lib()
    w = synth.quantized_weights(2)
    model = QuantizedNnue(w, device=local)
    pos = synth.positions(BATCH, 1 + rank)
    n_idx = len(pos.indices)
    idx = as_device(pos.indices, dev)
    off = as_device(pos.offsets, dev)
    scores = torch.empty(BATCH, dtype=torch.int32, device=dev)
    ws = model.workspace(BATCH)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    h = model.handle

    def step():
        check(L.cnnue_q_bucket_sort(h, off.data_ptr(), n_idx, BATCH, ws.data_ptr(), ws.numel(), sp), "sort")
        mid = torch.cuda.Event(enable_timing=True)
        mid.record(stream)
        check(L.cnnue_q_forward_sorted(h, idx.data_ptr(), n_idx, off.data_ptr(), BATCH, scores.data_ptr(),
                                       ws.data_ptr(), ws.numel(), sp), "forward")
        return mid

    # correctness of the timed configuration, once, before timing
    for _ in range(max(args.warmup, 3)):
        flush.fill_(rank + 1)
        step()
    torch.cuda.synchronize(dev)
    st = C.c_int(0)
    check(L.cnnue_read_status(ws.data_ptr(), sp, C.byref(st)), "status")
    check(st.value, "kernel status")

    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.3)
    starts, mids, ends = [], [], []
    for _ in range(args.steps):
        flush.fill_(1)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        m = step()
        e.record(stream)
        starts.append(s)
        mids.append(m)
        ends.append(e)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    kern_ms = [m.elapsed_time(e) for m, e in zip(mids, ends)]
    total_ms = sum(step_ms)
    kern_avg = sum(kern_ms) / len(kern_ms)

    # ---- e2e through the pipelined host-buffer C ABI (cnnue_q_ctx_*) ----------
    # Every step copies its indices and offsets from pinned host memory to the
    # device and its scores back; two steps are in flight, so one step's
    # copies overlap the previous step's kernels.  The L2 is flushed before
    # every step's kernels, on the stream the step runs on.  Timed by the host
    # clock from the first submit to the last completed wait.
    h_idx = torch.empty(n_idx, dtype=torch.int16, pin_memory=True).numpy().view(np.uint16)
    h_off = torch.empty(len(pos.offsets), dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    h_outs = [torch.empty(BATCH, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
    h_idx[:] = pos.indices
    h_off[:] = pos.offsets
    pipe = model.pipeline(BATCH, n_idx)

    def e2e_run(k_steps):
        pending = []
        for k in range(k_steps):
            if len(pending) == 2:
                check(pipe.wait(pending.pop(0)), "pipelined step status")
            xs = torch.cuda.ExternalStream(pipe.next_stream(), device=dev)
            with torch.cuda.stream(xs):
                flush.fill_(k + 2)
            pending.append(pipe.submit(h_idx, h_off, h_outs[k % 2]))
        for t in pending:
            check(pipe.wait(t), "pipelined step status")

    e2e_run(max(args.warmup, 3))
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    e2e_run(args.steps)
    e2e_avg = 1e3 * (time.perf_counter() - t0) / args.steps
    ok = bool(np.array_equal(h_outs[0], scores.cpu().numpy()) and np.array_equal(h_outs[1], scores.cpu().numpy()))
    pipe.close()

    # ---- max over ranks --------------------------------------------------------
    stats = torch.tensor([total_ms, kern_avg, e2e_avg, 0.0 if ok else 1.0], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total_ms, kern_avg, e2e_avg, bad = stats.tolist()
    if bad:
        raise RuntimeError("host-buffer scores differ from device-resident scores")

    if rank == 0:
        ms_per_step = total_ms / args.steps
        value = world * BATCH / (ms_per_step / 1e3)
        peak, peak_kind = measured_hbm_peak()
        alg = algorithmic_bytes(BATCH, n_idx)
        achieved = alg / (kern_avg / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": BATCH, "global_batch": world * BATCH,
                       "l2": "flushed between steps (256 MiB write)",
                       "parallelism": f"dp{world} (independent batches, no collective)"},
            "e2e": {"value": world * BATCH / (e2e_avg / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": int(h_idx.nbytes + h_off.nbytes), "d2h_bytes_per_step": int(h_outs[0].nbytes),
                    "api": "cnnue_q_forward_host_async + cnnue_q_ctx_wait, two steps in flight, L2 flushed before "
                           "every step, host clock"},
            "gpu_launches": 5 * args.steps,  # bucket count/scan/scatter, gather + pack, tensor-core stacks
            "roofline": {"bound": "hbm", "kernel": "q_gather_kernel + q_stack_tc_kernel", "achieved": achieved,
                         "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": committed_traffic(), "algorithmic_bytes_per_launch": alg,
                         "kernel_ms": kern_avg},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            from chineseai_b200 import synth as _s  # noqa: F401
            threads = cpu_threads()
            reps, el = cpu_time_batches(w, pos, threads, args.cpu_seconds, 2)
            line["cpu_baseline"] = {"value": reps * BATCH / el, "unit": UNIT, "cores": threads, "kind": "port",
                                    "sample": f"{reps} x full {BATCH}-position batch, {threads} OpenMP threads, "
                                              f"{el:.1f} s, CPU {cpu_cpu_model()}"}
        print(json.dumps(line), flush=True)
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# training-step workload (--workload train; not the headline line)
# ---------------------------------------------------------------------------
TRAIN_BATCH = 16384
TRAIN_METRIC = "training samples/sec (HalfKA FT 11340x1024, batch 16384 per GPU, data parallel)"


def run_train(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    from chineseai_b200 import synth, train
    from chineseai_b200.quantized import as_device

    tr = train.Trainer(train.init_params(3), device=local, group=pg.group.WORLD if pg else None,
                       ft_chunks=args.ft_chunks, shard=not args.no_shard)
    pos = synth.positions(TRAIN_BATCH, 1 + rank)
    t = torch.from_numpy(train.targets(TRAIN_BATCH, 100 + rank)).to(dev)
    idx, off = as_device(pos.indices, dev), as_device(pos.offsets, dev)
    n_idx = len(pos.indices)
    stream = torch.cuda.current_stream(dev)

    def step():
        tr.step(idx, n_idx, off, TRAIN_BATCH, t)  # overlapped exchange when world > 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if tr.status() != 0:
        raise RuntimeError("training kernels reported bad input")
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.3)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for k in range(args.steps):
        evs[k][0].record(stream)
        step()
        evs[k][1].record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    total = sum(e[0].elapsed_time(e[1]) for e in evs)

    # Phase times outside the timed region: the local forward + backward and
    # Adam alone, and a plain sum all-reduce of the whole gradient (bus
    # bandwidth per rank count).
    fb = _device_loop(lambda: tr.forward_backward(idx, n_idx, off, TRAIN_BATCH, t), args.steps, dev, stream)
    ad = _device_loop(lambda: train.lib().cnnue_t_adam(tr.params.data_ptr(), tr.m.data_ptr(), tr.v.data_ptr(),
                                                       tr.grads.data_ptr(), tr.shadow.data_ptr(), 0.0, 1e-12, 0.9,
                                                       0.999, 1e-8, 1, None, stream.cuda_stream), args.steps, dev,
                      stream)
    ar = rsag = 0.0
    if pg:
        scratch = torch.zeros_like(tr.grads)
        pg.barrier()
        ar = _device_loop(lambda: pg.all_reduce(scratch, op=pg.ReduceOp.SUM), args.steps, dev, stream)
        # the sharded exchange's collectives alone: FT fp32 reduce-scatter + bf16 all-gather
        ft = train.OFF_W1
        part = ft // world
        sh = torch.zeros(ft, dtype=torch.bfloat16, device=dev)

        def rs_ag():
            pg.reduce_scatter_tensor(scratch[:part], scratch[:ft], op=pg.ReduceOp.SUM)
            pg.all_gather_into_tensor(sh, sh[:part])

        pg.barrier()
        rsag = _device_loop(rs_ag, args.steps, dev, stream)
        del scratch, sh
    stats = torch.tensor([total, fb, ar, ad, rsag], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total, fb, ar, ad, rsag = stats.tolist()
    fb, ar, ad, rsag = fb / args.steps, ar / args.steps, ad / args.steps, rsag / args.steps
    loss = float(tr.loss.item())
    if rank == 0:
        ms = total / args.steps
        grad_bytes = 4 * train.param_count()
        line = {
            "metric": TRAIN_METRIC, "value": world * TRAIN_BATCH / (ms / 1e3), "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16/fp32",
            "data": "synthetic",
            "config": {"workload": "HalfKA training step: bf16 FT gather, pack, 16 bucket fp32 stacks (L1 on "
                                   "tcgen05), MSE(sigmoid(s/400), t), atomic-free FT backward, Adam; N > 1: "
                                   "stack gradients all-reduced beside the FT backward, FT gradient "
                                   + ("all-reduced" if args.no_shard else
                                      "reduce-scattered, Adam on this rank's FT shard, bf16 FT shadow "
                                      "all-gathered"),
                       "batch_per_gpu": TRAIN_BATCH, "global_batch": world * TRAIN_BATCH,
                       "parallelism": f"dp{world}", "grad_bytes": grad_bytes, "ft_chunks": args.ft_chunks,
                       "ft_exchange": "all-reduce" if args.no_shard else "sharded"},
            "phases_ms": {"forward_backward_alone": fb, "allreduce_alone": ar, "adam_alone": ad,
                          "rs_ag_alone": rsag, "exposed_exchange_and_adam": ms - fb},
            "allreduce_busbw_gbs": (2 * (world - 1) / world * grad_bytes / (ar / 1e3) / 1e9) if world > 1 else None,
            "loss": loss, "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# ResNet policy/value inference (--workload resnet; not the headline line)
# ---------------------------------------------------------------------------
RN_BATCH = 1024
RN_FLOPS_PER_BOARD = (90 * 128 * 135 * 2 + 20 * 90 * 128 * 1152 * 2 + 2 * 180 * 2086 + 90 * 128 * 3 * 2
                      + 2 * 90 * 256 + 2 * 256)


def measured_bf16_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops")), "measured"
    except Exception:
        return 1590.0, "fallback"


def _device_loop(step, steps, dev, stream):
    """Events around each step on `stream`; returns the summed milliseconds."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize(dev)
    return sum(a.elapsed_time(b) for a, b in evs)


def run_resnet(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    from chineseai_b200 import resnet

    w = resnet.ResNetWeights.synthetic(5)
    model = resnet.ResNetModel(w, device=local)
    planes = resnet.synthetic_planes(RN_BATCH, 6 + rank)
    d_planes = torch.from_numpy(planes.view(np.int16)).to(dev)
    h_planes = torch.from_numpy(planes.view(np.int16)).pin_memory()
    h_probs = torch.empty((RN_BATCH, resnet.MOVES), dtype=torch.float32).pin_memory()
    h_value = torch.empty(RN_BATCH, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        model.forward(d_planes)

    def step_e2e():
        d_planes.copy_(h_planes, non_blocking=True)
        probs, _, value = model.forward(d_planes)
        h_probs.copy_(probs, non_blocking=True)
        h_value.copy_(value, non_blocking=True)

    for _ in range(args.warmup):
        step()
        step_e2e()
    torch.cuda.synchronize(dev)
    if model.read_status() != 0:
        raise RuntimeError("resnet kernels reported a timeout")
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    sampler.start()
    time.sleep(0.3)
    total = 0.0
    for _ in range(args.steps):
        flush.zero_()
        total += _device_loop(step, 1, dev, stream)
    clocks = sampler.stop()
    e2e_total = _device_loop(step_e2e, args.steps, dev, stream)
    stats = torch.tensor([total, e2e_total], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total, e2e_total = stats.tolist()
    if rank == 0:
        ms = total / args.steps
        peak, peak_kind = measured_bf16_peak()
        achieved = RN_FLOPS_PER_BOARD * RN_BATCH / (ms / 1e3) / 1e12
        line = {
            "metric": "AlphaZero ResNet leaf evaluations/sec (policy 2086 + value, batch 1024)",
            "value": world * RN_BATCH / (ms / 1e3), "unit": "boards/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": "ResNet 10x128 (stem 3x3 15->128, 10 residual blocks), policy FC 180->2086 + "
                                   "softmax, value 90->256->1 tanh; input bf16 [1024][15][10][9]",
                       "batch_per_gpu": RN_BATCH, "parallelism": f"replicas{world}",
                       "l2": "flushed (256 MiB write) before each timed step"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "scope": "whole forward (21 tcgen05 convs + heads), algorithmic FLOPs"},
            "e2e": {"value": world * RN_BATCH / (e2e_total / args.steps / 1e3), "unit": "boards/s",
                    "h2d_bytes_per_step": planes.nbytes,
                    "d2h_bytes_per_step": RN_BATCH * resnet.MOVES * 4 + RN_BATCH * 4},
            "clocks": clocks, "gpu_launches": 25 * args.steps,  # pack + 21 convs + 1x1 convs + FC/value + softmax
        }
        if not args.no_cpu_baseline:
            import oracle
            sample = 8
            t0 = time.time()
            reps = 0
            while time.time() - t0 < min(args.cpu_seconds, 10.0) or reps == 0:
                oracle.rn_forward(w, planes[:sample])
                reps += 1
            el = time.time() - t0
            line["cpu_baseline"] = {"value": reps * sample / el, "unit": "boards/s", "cores": cpu_threads(),
                                    "kind": "port", "sample": f"{reps} x {sample} boards of the same batch"}
        print(json.dumps(line), flush=True)
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# Reference-native AZ-NNUE evaluation (--workload az; not the headline line)
# ---------------------------------------------------------------------------
AZ_POSITIONS = 65536


def run_az(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    from chineseai_b200 import az
    from chineseai_b200.quantized import as_device

    w = az.AzWeights.random(128, 20260807)
    model = az.AzModel(w, device=local)
    base = az.random_boards(4096, seed=1 + rank, keep=0.9)
    reps = AZ_POSITIONS // len(base)
    items0, offsets0 = az.node_lists(base)
    lens = np.diff(offsets0)
    items = np.tile(items0, reps)
    offsets = np.concatenate([[0], np.cumsum(np.tile(lens, reps))]).astype(np.uint32)
    side = np.tile((np.arange(len(base)) % 2).astype(np.uint8), reps)
    d_items, d_off, d_side = as_device(items, dev), as_device(offsets, dev), as_device(side, dev)
    acc = torch.empty((2 * AZ_POSITIONS, 128), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    h_items = torch.from_numpy(items.view(np.int32)).pin_memory()
    h_off = torch.from_numpy(offsets.view(np.int32)).pin_memory()
    h_wdl = torch.empty((AZ_POSITIONS, 3), dtype=torch.float32).pin_memory()
    h_q = torch.empty(AZ_POSITIONS, dtype=torch.float32).pin_memory()

    def step():
        model.refresh(d_items, d_off, out=acc)
        return model.value(acc, side=d_side)

    def step_e2e():
        d_items.copy_(h_items, non_blocking=True)
        d_off.copy_(h_off, non_blocking=True)
        wdl, q = step()
        h_wdl.copy_(wdl, non_blocking=True)
        h_q.copy_(q, non_blocking=True)

    for _ in range(args.warmup):
        step()
        step_e2e()
    torch.cuda.synchronize(dev)
    if model.read_status() != 0:
        raise RuntimeError("az kernels reported bad input")
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    sampler.start()
    time.sleep(0.3)
    total = refresh_ms = 0.0
    for _ in range(args.steps):
        flush.zero_()
        refresh_ms += _device_loop(lambda: model.refresh(d_items, d_off, out=acc), 1, dev, stream)
        flush.zero_()
        total += _device_loop(step, 1, dev, stream)
    clocks = sampler.stop()
    e2e_total = _device_loop(step_e2e, args.steps, dev, stream)
    stats = torch.tensor([total, e2e_total, refresh_ms], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total, e2e_total, refresh_ms = stats.tolist()
    if rank == 0:
        ms = total / args.steps
        r_ms = refresh_ms / args.steps
        n_items = len(items)
        alg = (2 * AZ_POSITIONS + 6 * n_items) * 128 * 4 + n_items * 4 + offsets.nbytes + 2 * AZ_POSITIONS * 128 * 4
        peak, peak_kind = measured_hbm_peak()
        achieved = alg / (r_ms / 1e3) / 1e9
        line = {
            "metric": "AZ-NNUE evaluations/sec (trunk refresh of both perspectives + value head, H=128)",
            "value": world * AZ_POSITIONS / (ms / 1e3), "unit": "positions/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "AzNnue::random(128, 20260807); 65,536 synthetic boards (~29 pieces), "
                                   "refresh bit-identical to the reference, value head WDL",
                       "batch_per_gpu": AZ_POSITIONS, "parallelism": f"replicas{world}",
                       "l2": "flushed (256 MiB write) before each timed step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "scope": "az_list_kernel (refresh), algorithmic bytes; rows are L2-resident"},
            "e2e": {"value": world * AZ_POSITIONS / (e2e_total / args.steps / 1e3), "unit": "positions/s",
                    "h2d_bytes_per_step": items.nbytes + offsets.nbytes,
                    "d2h_bytes_per_step": AZ_POSITIONS * 16},
            "clocks": clocks, "gpu_launches": 2 * args.steps,
        }
        if not args.no_cpu_baseline:
            import oracle
            tensors = w.tensors()
            sample = 4096
            s_off = offsets[: 2 * sample + 1]
            s_items = items[: s_off[-1]]
            t0 = time.time()
            n_rep = 0
            while time.time() - t0 < min(args.cpu_seconds, 10.0) or n_rep == 0:
                _, a = oracle.az_refresh(tensors, 128, s_items, s_off)
                oracle.az_value(tensors, 128, a.reshape(sample, 2, 128)[np.arange(sample), side[:sample]])
                n_rep += 1
            el = time.time() - t0
            line["cpu_baseline"] = {"value": n_rep * sample / el, "unit": "positions/s", "cores": 1,
                                    "kind": "port", "sample": f"{n_rep} x {sample} positions, single thread"}
        print(json.dumps(line), flush=True)
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# fp32 HalfKA forward (--workload fp32) and incremental update (--workload update)
# ---------------------------------------------------------------------------
F32_BATCH = 4096
F32_STACK_BYTES = 8 * (16 * 512 + 16 + 32 * 16 + 32 + 32 + 1) * 4 + 256 * 4


def _dist_init(local):
    import torch
    if dist_env()[1] == 1:
        return None
    import datetime

    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist


def _timed_steps(step, steps, dev, stream, flush):
    """Per step: L2 flush (not timed), then the step between CUDA events."""
    import torch
    total = 0.0
    for _ in range(steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        total += a.elapsed_time(b)
    return total


def run_fp32(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = _dist_init(local)
    from chineseai_b200 import synth
    from chineseai_b200.fp32 import FloatNnue
    from chineseai_b200.quantized import as_device

    w = synth.float_weights(2)
    model = FloatNnue(w, device=local)
    pos = synth.positions(F32_BATCH, 1 + rank)
    n_idx = len(pos.indices)
    idx, off = as_device(pos.indices, dev), as_device(pos.offsets, dev)
    out = torch.empty(F32_BATCH, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    h_idx = torch.from_numpy(pos.indices.view(np.int16)).pin_memory()
    h_off = torch.from_numpy(pos.offsets.view(np.int32)).pin_memory()
    h_out = torch.empty(F32_BATCH, dtype=torch.float32).pin_memory()

    def step():
        model.forward(idx, off, F32_BATCH, out=out, check_status=False)

    def step_e2e():
        idx.copy_(h_idx, non_blocking=True)
        off.copy_(h_off, non_blocking=True)
        step()
        h_out.copy_(out, non_blocking=True)

    for _ in range(max(args.warmup, 3)):
        step_e2e()
    model.forward(idx, off, F32_BATCH, out=out)  # checks the kernel status once
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    sampler.start()
    time.sleep(0.3)
    total = _timed_steps(step, args.steps, dev, stream, flush)
    clocks = sampler.stop()
    e2e_total = _timed_steps(step_e2e, args.steps, dev, stream, flush)
    stats = torch.tensor([total, e2e_total], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total, e2e_total = stats.tolist()
    if rank == 0:
        ms = total / args.steps
        alg = n_idx * 256 * 4 + n_idx * 2 + pos.offsets.nbytes + F32_BATCH * 4 + F32_STACK_BYTES
        peak, peak_kind = measured_hbm_peak()
        achieved = alg / (ms / 1e3) / 1e9
        line = {
            "metric": "fp32 HalfKA NNUE evals/sec (batch 4096)", "value": world * F32_BATCH / (ms / 1e3),
            "unit": "evals/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "fp32 HalfKA forward: FT 11340x256 N(0,0.01) per perspective, 2-32 unique "
                                   "sorted indices, CReLU, bucket=(n0-1)/4 of 8 stacks 512->16->32->1",
                       "batch_per_gpu": F32_BATCH, "parallelism": f"replicas{world}",
                       "l2": "flushed (256 MiB write) before each timed step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "kernel": "f_fused_kernel",
                         "scope": "whole forward (one kernel): gathered fp32 rows, indices, offsets, outputs, "
                                  "stack weights once; the 11.6 MB table is L2-resident after the first rows"},
            "e2e": {"value": world * F32_BATCH / (e2e_total / args.steps / 1e3), "unit": "evals/s",
                    "h2d_bytes_per_step": int(pos.indices.nbytes + pos.offsets.nbytes),
                    "d2h_bytes_per_step": F32_BATCH * 4},
            "clocks": clocks, "gpu_launches": args.steps,  # f_fused_kernel
        }
        if not args.no_cpu_baseline:
            import oracle
            t0 = time.time()
            reps = 0
            while time.time() - t0 < min(args.cpu_seconds, 10.0) or reps == 0:
                oracle.f_forward(w, pos)
                reps += 1
            el = time.time() - t0
            line["cpu_baseline"] = {"value": reps * F32_BATCH / el, "unit": "evals/s", "cores": 1, "kind": "port",
                                    "sample": f"{reps} x the 4096-position batch, one thread"}
        print(json.dumps(line), flush=True)
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_update(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = _dist_init(local)
    from chineseai_b200 import synth
    from chineseai_b200._lib import check, lib
    from chineseai_b200.quantized import QuantizedNnue, as_device

    L = lib()
    w = synth.quantized_weights(2)
    model = QuantizedNnue(w, device=local)
    ub = synth.update_batch(BATCH, 1 + rank)
    n = ub.n
    parent = as_device(ub.parent, dev)
    flags, c0 = as_device(ub.flags, dev), as_device(ub.count0, dev)
    rem, add = as_device(ub.rem, dev), as_device(ub.add, dev)
    ro, ao = as_device(ub.rem_offsets, dev), as_device(ub.add_offsets, dev)
    child = torch.empty((n, 2, 1024), dtype=torch.int16, device=dev)
    scores = torch.empty(n, dtype=torch.int32, device=dev)
    ws = model.workspace(n)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    pinned = {k: torch.from_numpy(np.ascontiguousarray(getattr(ub, k)).view(
        {1: np.int8, 2: np.int16, 4: np.int32}[getattr(ub, k).dtype.itemsize])).pin_memory()
        for k in ("flags", "rem", "rem_offsets", "add", "add_offsets", "count0")}
    dst = {"flags": flags, "rem": rem, "rem_offsets": ro, "add": add, "add_offsets": ao, "count0": c0}
    h_scores = torch.empty(n, dtype=torch.int32).pin_memory()

    def step():
        check(L.cnnue_q_update(model.handle, parent.data_ptr(), flags.data_ptr(), rem.data_ptr(), len(ub.rem),
                               ro.data_ptr(), add.data_ptr(), len(ub.add), ao.data_ptr(), c0.data_ptr(), n,
                               child.data_ptr(), scores.data_ptr(), ws.data_ptr(), ws.numel(), sp), "update")

    def step_e2e():
        for k, t in pinned.items():
            dst[k].view(t.dtype).copy_(t, non_blocking=True)
        step()
        h_scores.copy_(scores, non_blocking=True)

    for _ in range(max(args.warmup, 3)):
        step_e2e()
    torch.cuda.synchronize(dev)
    check(model.read_status(ws), "update kernel status")
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    sampler.start()
    time.sleep(0.3)
    total = _timed_steps(step, args.steps, dev, stream, flush)
    clocks = sampler.stop()
    e2e_total = _timed_steps(step_e2e, args.steps, dev, stream, flush)
    stats = torch.tensor([total, e2e_total], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total, e2e_total = stats.tolist()
    if rank == 0:
        ms = total / args.steps
        rows = len(ub.rem) + len(ub.add)
        list_bytes = sum(np.asarray(getattr(ub, k)).nbytes for k in dst)
        alg = n * 4096 * 2 + rows * 2048 + list_bytes + n * 4 + STACK_BYTES
        peak, peak_kind = measured_hbm_peak()
        achieved = alg / (ms / 1e3) / 1e9
        line = {
            "metric": "quantised incremental update + stack evals/sec (batch 64K)",
            "value": world * n / (ms / 1e3), "unit": "evals/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int16/int8", "data": "synthetic",
            "config": {"workload": "65,536 int16 parent accumulators [2][1024] U[-2000,2000]; per perspective 1-2 "
                                   "removed and 1-3 added rows, 5% full refreshes of 2-32 rows; then the pairwise "
                                   "pack and the 16 int8 bucket stacks", "batch_per_gpu": n,
                       "parallelism": f"replicas{world}", "l2": "flushed (256 MiB write) before each timed step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "scope": "cnnue_q_update (one kernel): parent read + child write (8 KB per position), "
                                  "2 KB per added/removed row, the lists, scores, stack weights once"},
            "e2e": {"value": world * n / (e2e_total / args.steps / 1e3), "unit": "evals/s",
                    "h2d_bytes_per_step": int(list_bytes), "d2h_bytes_per_step": n * 4,
                    "note": "parents and children stay on the device (the search's node arena); the step's "
                            "delta lists go up and its scores come back"},
            "clocks": clocks, "gpu_launches": args.steps,
        }
        if not args.no_cpu_baseline:
            import oracle
            sample = synth.update_batch(8192, 1 + rank)
            t0 = time.time()
            reps = 0
            while time.time() - t0 < min(args.cpu_seconds, 10.0) or reps == 0:
                oracle.q_update(w, sample, n_threads=cpu_threads())
                reps += 1
            el = time.time() - t0
            line["cpu_baseline"] = {"value": reps * sample.n / el, "unit": "evals/s", "cores": cpu_threads(),
                                    "kind": "port", "sample": f"{reps} x 8192 updates (same generator), "
                                                              "all host threads"}
        print(json.dumps(line), flush=True)
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# AZ-NNUE training step (--workload az-train; not the headline line)
# ---------------------------------------------------------------------------
AZ_TRAIN_BATCH = 1024  # the reference's default batch (src/az_loop_config.rs:115)
AZ_TRAIN_CAPS = (40, 96, 96)  # fixed per-row widths: features, policy moves, threats


def adam_traffic(n_params: int):
    """DRAM bytes per AdamW launch from the committed ncu capture
    (profiles/adamw_vec4_kernel.json), scaled to n_params."""
    try:
        with open(os.path.join(ROOT, "profiles", "adamw_vec4_kernel.json")) as f:
            d = json.load(f)
        return int(d["dram_bytes_per_launch"] * n_params / d["params"])
    except Exception:
        return None


def run_az_train(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    from chineseai_b200 import az, az_train

    B = AZ_TRAIN_BATCH
    w = az.AzWeights.random(128, 20260807)
    samples = az_train.random_samples(4 * B, seed=1 + rank)
    t0 = time.time()
    batches = [az_train.pack_batch(samples, np.arange(k * B, (k + 1) * B), caps=AZ_TRAIN_CAPS, fixed=True,
                                   compact=True) for k in range(4)]
    pack_ms = (time.time() - t0) / 4 * 1e3
    tr = az_train.AzTrainer(w, lr=1e-3, device=local, graph=True, group=pg.group.WORLD if pg else None)
    for i in range(max(args.warmup, 3)):
        tr.step(batches[i % 4])
    # kernels of one step: a profiled eager step of a twin trainer (outside the timed region)
    from torch.profiler import ProfilerActivity, profile
    twin = az_train.AzTrainer(w, lr=1e-3, device=local)  # single-rank twin: counts kernels, no collective
    twin.step(batches[0])
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        twin.step(batches[1])
        torch.cuda.synchronize(dev)
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ours_per_step = sum(1 for n in names if "cnnue" in n)
    all_per_step = sum(1 for n in names if not n.startswith("Memcpy") and not n.startswith("Memset"))
    del twin
    stream = torch.cuda.current_stream(dev)
    # device-resident: replays of the captured step on a batch already in HBM
    tr.to_device(batches[0])
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    sampler.start()
    time.sleep(0.3)
    def device_step():
        tr._graph.replay()  # with N > 1 the graph holds the NCCL exchange and AdamW too
        if tr.world > 1 and not tr._in_graph_exchange():
            tr._exchange(tr._graph_out, read=False)
            tr._adamw()

    total = _device_loop(device_step, args.steps, dev, stream)
    clocks = sampler.stop()
    # end to end: AzTrainer.step on host batches (pinned staging + H2D, metrics back)
    e2e_total = _device_loop(lambda: tr.step(batches[np.random.randint(4)]), args.steps, dev, stream)
    # AdamW alone (the one kernel with a clean roofline: 28 bytes per parameter)
    adam_ms = _device_loop(
        lambda: az_train.lib().cnnue_adamw(tr.flat.data_ptr(), tr.m.data_ptr(), tr.v.data_ptr(),
                                           tr.grad.data_ptr(), tr.n_params, 1e-9, 0.9, 0.999, 1e-8, 0.0,
                                           tr.step_count + 1, stream.cuda_stream), args.steps, dev, stream)
    stats = torch.tensor([total, e2e_total, adam_ms], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total, e2e_total, adam_ms = stats.tolist()
    if rank == 0:
        ms = total / args.steps
        a_ms = adam_ms / args.steps
        peak, peak_kind = measured_hbm_peak()
        adam_bytes = 28 * tr.n_params
        achieved = adam_bytes / (a_ms / 1e3) / 1e9
        b0 = batches[0]
        h2d = sum(np.asarray(getattr(b0, f.name)).nbytes for f in dataclasses.fields(b0)
                  if getattr(b0, f.name) is not None)
        line = {
            "metric": "AZ-NNUE training samples/sec (forward, WDL + masked policy CE, backward, AdamW; H=128)",
            "value": world * B / (ms / 1e3), "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "AzNnue::random(128, 20260807); batch 1024 synthetic self-play samples "
                                   "(random boards, pseudo moves, gamma visit targets), fixed widths "
                                   f"{AZ_TRAIN_CAPS}, compact batches (lookup indices rebuilt on the GPU); "
                                   "one CUDA-graph step", "batch_per_gpu": B,
                       "parallelism": f"dp{world}" if world > 1 else "dp1", "host_pack_ms_per_batch": pack_ms,
                       "l2": "not flushed: the step's inputs and parameters (~33 MB) are L2-sized"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": adam_traffic(tr.n_params),
                         "scope": f"adamw_vec4_kernel alone: 28 B x {tr.n_params} parameters per launch, "
                                  f"{a_ms * 1e3:.1f} us"},
            "e2e": {"value": world * B / (e2e_total / args.steps / 1e3), "unit": "samples/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 31 * 4},
            "clocks": clocks, "gpu_launches": ours_per_step * args.steps,
            "kernels_per_step": {"ours": ours_per_step, "all": all_per_step},
        }
        if not args.no_cpu_baseline:
            import oracle
            from oracle import az_train_ref
            torch.set_num_threads(cpu_threads())
            sample = 64
            sb = az_train.pack_batch(samples, np.arange(sample))
            tensors = w.tensors()
            t0 = time.time()
            n_rep = 0
            while time.time() - t0 < min(args.cpu_seconds, 15.0) or n_rep == 0:
                _, grads = az_train_ref.gradients(tensors, sb, dtype=torch.float32)
                flat_p = np.concatenate([t.reshape(-1) for t in tensors]).astype(np.float32)
                flat_g = np.concatenate([g.reshape(-1) for g in grads]).astype(np.float32)
                oracle.adamw(flat_p, np.zeros_like(flat_p), np.zeros_like(flat_p), flat_g, 1e-3, step=1)
                n_rep += 1
            el = time.time() - t0
            line["cpu_baseline"] = {"value": n_rep * sample / el, "unit": "samples/s", "cores": cpu_threads(),
                                    "kind": "port",
                                    "sample": f"{n_rep} steps of {sample} samples: torch-CPU restatement "
                                              "(fp32 autograd) + the oracle's AdamW"}
        print(json.dumps(line), flush=True)
    tr.close()  # releases the captured graph (it may hold NCCL calls)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# Wide-batch AlphaZero search (--workload mcts; not the headline line)
# ---------------------------------------------------------------------------
MCTS_ROOTS = 4096
MCTS_SIMS = 64
START_FEN = "rnbakabnr/9/1c5c1/p1p1p1p1p/9/9/P1P1P1P1P/1C5C1/9/RNBAKABNR w - - 0 1"


def playout_roots(n: int, seed: int):
    """The start position and positions after 1-40 random legal moves from it."""
    from chineseai_b200 import az, mcts
    rng = np.random.default_rng(seed)
    b0, s0 = az.board_from_fen(START_FEN)
    boards, sides = [b0], [s0]
    while len(boards) < n:
        b, side = b0.copy(), s0
        for _ in range(int(rng.integers(1, 41))):
            moves = mcts.legal_moves(b, side)
            if len(moves) == 0 or not (b == -1).any() or not (b == 1).any():
                break
            frm, to = moves[rng.integers(len(moves))]
            b[to], b[frm] = b[frm], 0
            side = 1 - side
        if (b == -1).any() and (b == 1).any() and len(mcts.legal_moves(b, side)):
            boards.append(b)
            sides.append(side)
    return np.array(boards, np.int8), np.array(sides, np.uint8)


def run_mcts(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    from chineseai_b200 import az, mcts

    w = az.AzWeights.random(128, 20260807)
    model = az.AzModel(w, device=local)
    boards, sides = playout_roots(MCTS_ROOTS, seed=1 + rank)
    search = mcts.Search(model, w)
    lim = mcts.default_limits(MCTS_SIMS)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(1, args.warmup // 3)):  # the timed shape: trees and buffers reach their size here
        search.run(boards, sides, lim, stream=stream.cuda_stream)
    sampler = ClockSampler(local)
    if pg:
        pg.barrier()
    sampler.start()
    time.sleep(0.3)
    evals = []
    box = {}

    def one():
        box["e"] = search.run(boards, sides, lim, stream=stream.cuda_stream)

    steps = max(1, min(args.steps, 3))
    total = 0.0
    for _ in range(steps):
        total += _device_loop(one, 1, dev, stream)
        evals.append(box["e"])
    clocks = sampler.stop()
    st = search.stats()
    stats = torch.tensor([total], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total = stats.item()
    if rank == 0:
        ms = total / steps
        ev = float(np.mean(evals))
        line = {
            "metric": "AZ wide-batch search: network leaf evaluations/sec (4096 roots x 64 simulations, H=128)",
            "value": world * ev / (ms / 1e3), "unit": "evals/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "AzNnue::random(128, 20260807); 4096 roots (start position + random legal "
                                   "playouts of 1-40 plies), 64 simulations each, AzSearchLimits defaults; "
                                   "roots in two halves whose GPU leaf batches alternate (one half is selected while the other is evaluated)", "roots_per_gpu": MCTS_ROOTS,
                       "simulations": MCTS_SIMS, "parallelism": f"replicas{world}",
                       "phase_seconds_last_search": st, "evaluations_per_search": ev,
                       "simulations_per_sec": world * MCTS_ROOTS * MCTS_SIMS / (ms / 1e3)},
            "roofline": None,
            "e2e": {"value": world * ev / (ms / 1e3), "unit": "evals/s",
                    "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                    "note": "the search is host-driven: value is already end to end"},
            "clocks": clocks, "gpu_launches": 4 * st["rounds"] * steps,
        }
        if not args.no_cpu_baseline:
            from oracle import mcts_ref
            th, ta = w.quant_flags()
            evr = mcts_ref.Evaluator(w.tensors(), 128, th, ta)
            t0 = time.time()
            n_ev = 0
            k = 0
            while time.time() - t0 < min(args.cpu_seconds, 15.0) or k == 0:
                srch = mcts_ref.Search(evr, boards[k % len(boards)], int(sides[k % len(sides)]), MCTS_SIMS).run()
                n_ev += sum(1 for n in srch.nodes if n["expanded"] and n["children"])
                k += 1
            el = time.time() - t0
            line["cpu_baseline"] = {"value": n_ev / el, "unit": "evals/s", "cores": 1, "kind": "port",
                                    "sample": f"{k} single-tree searches of {MCTS_SIMS} simulations: the "
                                              "oracle's search restatement with its C evaluator, one thread"}
        print(json.dumps(line), flush=True)
    search.close()
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ft-chunks", type=int, default=1, help="train, --no-shard: FT-gradient row chunks "
                    "all-reduced as they finish")
    ap.add_argument("--no-shard", action="store_true", help="train: all-reduce the FT gradient and run Adam over "
                    "everything on every rank, instead of the sharded exchange")
    ap.add_argument("--workload", choices=["eval", "fp32", "update", "train", "resnet", "az", "az-train", "mcts"],
                    default="eval",
                    help="eval: the headline quantised forward; fp32: the fp32 forward (batch 4096); "
                         "update: the incremental update + stack; train: the data-parallel training step; "
                         "resnet: AlphaZero ResNet leaf batch; az: reference-native AZ-NNUE evaluation; "
                         "az-train: the AZ-NNUE training step; mcts: the wide-batch AlphaZero search")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "train":
        return run_train(args)
    if args.workload == "resnet":
        return run_resnet(args)
    if args.workload == "az":
        return run_az(args)
    if args.workload == "az-train":
        return run_az_train(args)
    if args.workload == "mcts":
        return run_mcts(args)
    if args.workload == "fp32":
        return run_fp32(args)
    if args.workload == "update":
        return run_update(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
