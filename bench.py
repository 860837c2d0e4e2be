#!/usr/bin/env python
"""Benchmark: the wide-MLP data-parallel training step on B200.

Workload: Linear(4096,4096) -> ReLU -> Linear(4096,4096)
-> ReLU -> Linear(4096,10), cross_entropy, backward, gradient all-reduce
(mean, NCCL) across ranks, Sgd step lr=0.01; global batch 8192 split evenly
over the ranks (strong scaling).  Synthetic seeded data, reference init.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line on rank 0.  `value` is global training steps per second
measured on the device with inputs resident in HBM (CUDA events on the step's
stream, max over ranks); `e2e` is the same metric through the C-ABI host entry
point (fg_mlp_step_host) with the batch copied from pinned host memory and the
loss copied back every step.  At one GPU the line also carries `per_config`
(configs 1-4 and the lazy-Tensor front end at configs 1 and 5, each with its
roofline) and `cpu_baseline` (the oracle on one pinned host core, as the
single-threaded reference runs; an all-cores figure is attached as secondary).
`--impl reference` times the reference CPU arithmetic (the oracle port: the
Rust reference cannot be built here) on one pinned host core.
"""
from __future__ import annotations

import argparse
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

DIMS = (4096, 4096, 4096, 10)
GLOBAL_BATCH = 8192
LR = 0.01
X_SEED, LABEL_SEED = 13, 14
METRIC = "MLP train steps/s (wide MLP 4096-4096-4096-10, global batch 8192, fp32)"
WORKLOAD = "config5: wide MLP data-parallel training step (forward, cross_entropy, backward, allreduce-mean, SGD)"
GEMM_FLOPS_PER_STEP = 5 * (2 * 8192 * 4096 * 4096) + 3 * (2 * 8192 * 4096 * 10)


def env_dist():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# DRAM bytes per algorithmic flop of the config-5 forward GEMM launch, from one
# ncu capture of `python bench.py --config c5gemm --steps 1 --warmup 3`
# (dram__bytes_read.sum + dram__bytes_write.sum = 1.469e9 + 0.486e9 B over
# 2.749e11 flop; 16-deep k-blocks, segmented accumulation on);
# `roofline.traffic` is this times the flops of one launch.
GEMM_TRAFFIC_BYTES_PER_FLOP = 7.11e-3
# A timed region shorter than this runs at the burst clock; longer ones settle
# at the sustained (power-capped) clock.
SUSTAINED_AFTER_S = 2.0


# ---------------------------------------------------------------------------
# CPU side: the oracle (reference arithmetic) on a bounded sample
# ---------------------------------------------------------------------------
def _c5_params():
    from oracle import oracle as orc
    rng = orc.InitRng()
    ws, bs = [], []
    for i in range(len(DIMS) - 1):
        w, b = rng.linear(DIMS[i], DIMS[i + 1])
        ws.append(w)
        bs.append(b)
    return ws, bs


def cpu_step_sample(rows: int, threads: int, params=None):
    """Seconds of one C5 step restricted to `rows` batch rows on the oracle."""
    from oracle import oracle as orc
    from ferrograd_b200 import data
    orc.set_threads(threads)
    x, t = data.mlp_batch(rows, DIMS[0], DIMS[-1], X_SEED, LABEL_SEED)
    ws, bs = params if params is not None else _c5_params()
    t0 = time.perf_counter()
    orc.mlp_step(ws, bs, x, t, LR, want_grads=False)
    return time.perf_counter() - t0


class _Pinned:
    """Run the enclosed code on one host core (the reference is
    single-threaded: its generated loops run one at a time on the calling
    thread, src/device/cpu.rs:328-380)."""

    def __enter__(self):
        self.saved = os.sched_getaffinity(0)
        self.core = min(self.saved)
        os.sched_setaffinity(0, {self.core})
        return self

    def __exit__(self, *exc):
        os.sched_setaffinity(0, self.saved)


def _extrapolate(t_small: float, t_big: float, r_small: int, r_big: int) -> float:
    """Full-batch step seconds from two row samples: a step costs a fixed part
    (the SGD update and weight-only work) plus a part linear in the rows (every
    GEMM and the cross-entropy)."""
    per_row = max(t_big - t_small, 0.0) / (r_big - r_small)
    fixed = max(t_big - per_row * r_big, 0.0)
    return fixed + per_row * GLOBAL_BATCH


def cpu_baseline(target_s: float = 15.0):
    """The oracle on one pinned core (primary, as the reference runs), plus all
    host cores through OpenMP (secondary, labelled: not how the reference runs)."""
    params = _c5_params()
    with _Pinned() as pin:
        cpu_step_sample(8, 1, params)  # first touch of the weights
        t16 = cpu_step_sample(16, 1, params)
        t48 = cpu_step_sample(48, 1, params)
        per_row = max(t48 - t16, 1e-4) / 32
        rows = int(min(GLOBAL_BATCH, max(64, (target_s - t16) / per_row)))
        rows = max(64, rows // 16 * 16)
        tr = cpu_step_sample(rows, 1, params)
        core = pin.core
    step_s = _extrapolate(t16, tr, 16, rows)
    threads = os.cpu_count() or 1
    tp = cpu_step_sample(256, threads, params)
    tq = cpu_step_sample(1024, threads, params)
    mt_step_s = _extrapolate(tp, tq, 256, 1024)
    return {"value": 1.0 / step_s, "unit": "steps/s", "cores": 1, "kind": "port",
            "sample": (f"oracle (C restatement of the reference CPU arithmetic) pinned to host core "
                       f"{core}: one config-5 step on {rows} of {GLOBAL_BATCH} batch rows "
                       f"({tr:.2f} s) and on 16 rows ({t16:.2f} s), extrapolated linearly in the "
                       f"rows to the full batch (x{GLOBAL_BATCH / rows:.2f} on the per-row part)"),
            "secondary_all_cores": {
                "value": 1.0 / mt_step_s, "unit": "steps/s", "cores": threads,
                "note": "not how the reference runs: the oracle's output loops split over all "
                        "host cores by OpenMP; 256- and 1024-row samples "
                        f"({tp:.2f} s, {tq:.2f} s) extrapolated linearly"}}


def reference_arm(args):
    rank, world, _ = env_dist()
    if rank != 0:
        return 0
    params = _c5_params()
    rows_small, rows = 16, 64
    with _Pinned() as pin:
        cpu_step_sample(8, 1, params)
        t_small = statistics.median(cpu_step_sample(rows_small, 1, params) for _ in range(3))
        for _ in range(args.warmup):
            cpu_step_sample(rows, 1, params)
        times = [cpu_step_sample(rows, 1, params) for _ in range(args.steps)]
        core = pin.core
    step_s = _extrapolate(t_small, statistics.mean(times), rows_small, rows)
    value = 1.0 / step_s
    sample = (f"oracle port of the reference CPU arithmetic on 1 pinned host core ({core}; the "
              f"reference is single-threaded); each timed step is {rows} of {GLOBAL_BATCH} batch "
              f"rows of a config-5 step, extrapolated linearly in the rows to the full batch "
              f"(fixed part from {rows_small}-row samples, per-row part x{GLOBAL_BATCH / rows:.2f})")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform inputs, one-hot labels)",
            "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH, "dims": list(DIMS),
                       "parallelism": "none (CPU, 1 core)"},
            "cpu_baseline": {"value": value, "unit": "steps/s", "cores": 1, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "reference_note": "the Rust reference cannot be built here (no rustc/clang); the oracle "
                              "restates its arithmetic in C"}
    print(json.dumps(line), flush=True)
    return 0


def measure_tf32_tflops():
    """Dense TF32 tensor throughput of this GPU: torch fp32 matmul 8192^3 with
    TF32 allowed (cuBLAS), best of 10, CUDA events."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        g = torch.Generator(device="cuda").manual_seed(0)
        a = torch.randn((n, n), device="cuda", generator=g)
        b = torch.randn((n, n), device="cuda", generator=g)
        c = torch.empty((n, n), device="cuda")
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.path = tempfile.mktemp(suffix=".csv")
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path).read().splitlines()[1:]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                smax = float(parts[2].split()[0])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def our_arm(args):
    import datetime

    import torch
    import torch.distributed as dist

    from ferrograd_b200 import Communicator, CudaDevice, MlpTrainer, data, dp, mlp_init

    rank, world, local = env_dist()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    lo, hi = dp.shard_rows(GLOBAL_BATCH, rank, world)
    B = hi - lo

    x_full, t_full = data.mlp_batch(GLOBAL_BATCH, DIMS[0], DIMS[-1], X_SEED, LABEL_SEED)
    x = np.ascontiguousarray(x_full[lo:hi])
    t = np.ascontiguousarray(t_full[lo:hi])
    del x_full, t_full
    ws, bs = mlp_init(DIMS)  # seeded: identical on every rank

    comm = None
    if world > 1 and args.dp == "nccl":
        uid = dp.exchange_unique_id(dist, rank, Communicator.unique_id)
        comm = Communicator(rank, world, uid, timeout_ms=120000)
    dev = CudaDevice(local)
    tr = MlpTrainer(dev, DIMS, B, LR, ws, bs, comm=comm, use_graph=True)
    if world > 1 and args.dp == "peer":
        tr.shard_over_peers(rank, world, lambda h: dp.all_gather_bytes(dist, h, world),
                            dist.barrier, chunks=args.dp_chunks)
    tr.enable_gemm_timing(True)

    xp = torch.from_numpy(x).pin_memory()
    tp = torch.from_numpy(t).pin_memory()
    lossp = torch.zeros(1, dtype=torch.float32).pin_memory()
    stream = torch.cuda.ExternalStream(dev.stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        tt = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    # warm-up through the host entry point (fills the device input slots too)
    for _ in range(max(args.warmup, 3)):
        tr.step_host_ptr(xp.data_ptr(), tp.data_ptr(), lossp.data_ptr())
    first_loss = float(lossp.item())

    # ---- device-resident timing -------------------------------------------
    sampler = None
    if rank == 0:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        phys = int(vis.split(",")[local]) if vis and vis.split(",")[local].isdigit() else local
        sampler = ClockSampler(phys)
    if sampler:  # start sampling before the barrier so every rank enters the timed region together
        sampler.start()
        time.sleep(0.4)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = int(tr.launches_per_step)
    e0.record(stream)
    for _ in range(args.steps):
        tr.step()
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    gemms = tr.gemm_times()
    comms = tr.comm_times() if comm is not None else []

    # ---- end to end through the C ABI with host buffers --------------------
    # fg_mlp_step_host_next: each call copies the step's batch from pinned
    # host memory (uploaded by the copy engine while the previous step ran)
    # and reads the loss back; the first call uploads its own batch.
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tr.step_host_next_ptr(xp.data_ptr(), tp.data_ptr(), xp.data_ptr(), tp.data_ptr(),
                              lossp.data_ptr())
    e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
    last_loss = float(lossp.item())

    peaks, peak_src = load_peaks()
    region_s = ms * args.steps * 1e-3
    tf32_measured = measure_tf32_tflops() if rank == 0 else None
    gemm_ms = sum(g[0] for g in gemms)
    gemm_flops = sum(g[1] for g in gemms)
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    peak_key = "bf16_tflops" if region_s < SUSTAINED_AFTER_S else "bf16_tflops_sustained"
    tf32_peak = peaks[peak_key] / 2.0
    peak_3x = tf32_peak / 3.0
    per_launch_flops = gemm_flops / len(gemms) if gemms else 0
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak_3x, "unit": "TFLOP/s",
        "frac": (achieved / peak_3x) if achieved else None,
        "traffic": GEMM_TRAFFIC_BYTES_PER_FLOP * per_launch_flops if per_launch_flops else None,
        "kernel": "k_gemm3x (3xTF32 tcgen05, persistent, 128x256 tiles)",
        "achieved_basis": (f"2*M*N*K algorithmic flops / CUDA-event duration, averaged over the "
                           f"{len(gemms)} GEMM launches of the last timed step ({per_launch_flops:.3e} "
                           f"flop each)"),
        "peak_basis": (f"{peak_src} {peak_key} {peaks[peak_key]} / 2 (dense TF32 = half the bf16 "
                       f"rate) / 3 (3xTF32 issues three MMAs per product); {peak_key} because the "
                       f"timed region lasts {region_s:.3f} s (burst below {SUSTAINED_AFTER_S} s)"),
        "traffic_basis": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the config-5 forward "
                          f"GEMM launch per algorithmic flop ({GEMM_TRAFFIC_BYTES_PER_FLOP:.3g} B/flop, "
                          "profiles/gemm3x_c5_shapes_ncu.md) x the flops of one launch"),
        "frac_of_tf32_issue": ((3 * achieved) / tf32_peak) if achieved else None,
        "tf32_tflops_measured": tf32_measured,
        "frac_vs_measured_tf32": ((3 * achieved) / tf32_measured) if achieved and tf32_measured
        else None,
        "tf32_basis": "torch fp32 matmul 8192^3 with allow_tf32 (cuBLAS), best of 10, measured in "
                      "this run; frac_vs_measured_tf32 = 3 x achieved / it (three MMAs per product)",
    }
    # Parameters must stay identical across ranks (config 5): every rank hashes
    # its weights and biases after the last step; the digests are compared.
    from ferrograd_b200.dp import digests_agree, params_digest
    pw, pb = tr.params()
    digest = params_digest(list(pw) + list(pb))
    identical = digests_agree(dist, digest, world) if world > 1 else True
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: x uniform[0,1) seed 13, one-hot labels uniform 0..9 seed 14; "
                    "reference Linear::new init (seed-42 LCG Kaiming normal, zero bias)",
            "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH, "dims": list(DIMS),
                       "per_gpu_batch": B, "parallelism": f"dp{world}",
                       "gradient_exchange": (None if world == 1 else
                                             "NCCL all-reduce per layer bucket" if args.dp == "nccl"
                                             else f"peer-sharded: copy-engine reduce-scatter, owner "
                                                  f"reduce+SGD, copy-engine all-gather "
                                                  f"({args.dp_chunks} row chunks of layer 0)"),
                       "l2": "inputs larger than L2 (x shard + 2x64 MiB weights + residuals)",
                       "gemm": "3xTF32 tcgen05 (fp32-accurate)", "graph": "CUDA graph replay"},
            "roofline": roofline,
            "e2e": {"value": 1.0 / e2e_s, "unit": "steps/s",
                    "h2d_bytes_per_step": int(x.nbytes + t.nbytes), "d2h_bytes_per_step": 4,
                    "path": "fg_mlp_step_host_next: every step uploads a batch (x shard + "
                            "targets) from pinned host memory on a copy stream, overlapped with "
                            "the previous step's compute, and blocks on the loss read (wall "
                            "clock, max over ranks)"},
            "gemm_ms_last_step": [round(g[0], 4) for g in gemms],
            "allreduce_ms_mb_last_step": [[round(c[0], 4), round(c[1] / 2**20, 2)] for c in comms],
            "gpu_launches": launches0 * args.steps,
            "launches_per_step": launches0,
            "clocks": clocks,
            "loss_first_last": [first_loss, last_loss],
            "gemm_flops_per_step": GEMM_FLOPS_PER_STEP,
            "params_identical_across_ranks": bool(identical),
            "params_sha256_rank0": digest[:16],
        }
    if world > 1:
        barrier()
    tr.close()
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_per_config:
            line["per_config"] = per_config(peaks, peak_src)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        print(json.dumps(line), flush=True)
    return 0


PER_CONFIG = (("c1", 200, 5), ("c2", 20, 3), ("c3", 10, 3), ("c4", 20, 3), ("c1front", 100, 5),
              ("c5front", 10, 3), ("c2front", 20, 3), ("c4front", 20, 3))


def per_config(peaks, src):
    """Configs 1-4 and the lazy-Tensor front end (configs 1 and 5 through
    Linear / cross_entropy / backward / Sgd::step) at one GPU, each with its
    own roofline (and e2e for the training steps): one object per config.
    A config that fails reports its error instead of a value."""
    out = {}
    for name, iters, warm in PER_CONFIG:
        t0 = time.perf_counter()
        try:
            r = run_config(name, iters, warm, peaks, src)
            r.update({"steps": iters, "warmup": warm})
        except Exception as e:  # one failing leg must not lose the headline line
            r = {"error": repr(e)[:500]}
        r["wall_s"] = round(time.perf_counter() - t0, 2)
        out[name] = r
    return out


# ---------------------------------------------------------------------------
# Per-config kernel benchmarks (configs 1-4 of the workload list); the driver's
# headline line is config 5 above.  Each prints one JSON line.
# ---------------------------------------------------------------------------
def _event_time(fn, iters, flush=None):
    """Average ms of fn() on the current stream.

    Without `flush`, the iters calls are enqueued back to back between two
    CUDA events (the host's launch latency then overlaps the previous call
    instead of leaving the GPU idle inside the timed region).  With `flush`,
    each call is bracketed by its own events after an untimed flush.
    """
    import torch
    if flush is None:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / iters
    times = []
    for _ in range(iters):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.mean(times)


def _graph_time(fn, iters):
    """Average ms of fn() when `iters` calls are captured in one CUDA graph
    and replayed: kernels run back to back with no host launch cost between
    them (short kernels are otherwise bound by the Python call rate)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / iters
    del g
    return ms


def _step_roofline(flops, ms, peaks, src, bound):
    """Whole-step algorithmic flop rate against the 3xTF32 tensor peak (burst)."""
    tf = flops / (ms * 1e-3) / 1e12
    peak = peaks["bf16_tflops"] / 2 / 3
    return {"bound": bound, "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
            "traffic": None, "kernel": "whole step (all launches)",
            "peak_basis": f"{src} bf16_tflops (burst) / 2 (TF32) / 3 (3 MMAs per product)"}


def _hbm_roofline(nbytes, ms, peaks, src, kernel):
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": gbs / peaks["hbm_gbs"], "traffic": None, "kernel": kernel,
            "peak_basis": f"{src} hbm_gbs (copy bandwidth, burst)"}


def config_bench(args):
    peaks, src = load_peaks()
    iters, warm = args.steps, max(args.warmup, 3)
    line = run_config(args.config, iters, warm, peaks, src)
    line.update({"n_gpus": 1, "steps": iters, "warmup": warm, "dtype": "f32", "data": "synthetic"})
    print(json.dumps(line), flush=True)
    return 0


def run_config(config, iters, warm, peaks, src):
    """One JSON object for configuration `config` (c1-c4, c5gemm, c1front,
    c5front) on cuda:0."""
    import torch

    from ferrograd_b200 import CudaDevice, MlpTrainer, data, kernels, mlp_init
    from ferrograd_b200._lib import REDUCE_MAX, REDUCE_SUM

    flush_buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MiB > L2

    def flush():
        flush_buf.zero_()

    if config == "c1":
        dims, B = (784, 128, 10), 256
        x, t = data.mlp_batch(B, dims[0], dims[-1], 1, 2)
        tr = MlpTrainer(CudaDevice(0), dims, B, 0.01, *mlp_init(dims), use_graph=True)
        xp, tp = torch.from_numpy(x).pin_memory(), torch.from_numpy(t).pin_memory()
        lossp = torch.zeros(1).pin_memory()
        for _ in range(warm):
            tr.step_host_ptr(xp.data_ptr(), tp.data_ptr(), lossp.data_ptr())
        stream = torch.cuda.ExternalStream(tr.device.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(iters):
            tr.step()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        t0 = time.perf_counter()
        for _ in range(iters):
            tr.step_host_ptr(xp.data_ptr(), tp.data_ptr(), lossp.data_ptr())
        e2e_ms = (time.perf_counter() - t0) / iters * 1e3
        flops = 2 * B * (784 * 128 + 128 * 10) * 3 - 2 * B * 784 * 128  # no dX for the input
        line = {"metric": "config1 MLP train steps/s (784-128-10, batch 256)", "value": 1e3 / ms,
                "unit": "steps/s", "ms_per_step": ms, "launches_per_step": tr.launches_per_step,
                "e2e": {"value": 1e3 / e2e_ms, "unit": "steps/s",
                        "h2d_bytes_per_step": int(x.nbytes + t.nbytes), "d2h_bytes_per_step": 4},
                "flop_per_step": flops, "bound": "latency (launch-bound; CUDA graph replay)",
                "roofline": _step_roofline(flops, ms, peaks, src, "latency")}
    elif config == "c2":
        n = data.C2_N
        g = torch.Generator(device="cuda").manual_seed(3)
        a, b, c = (torch.randn(n, device="cuda", generator=g) for _ in range(3))
        out = torch.empty_like(a)
        fn = lambda: kernels.ew_fma_relu_scale(a, b, c, 0.5, out=out)  # noqa: E731
        for _ in range(warm):
            fn()
        ms = _event_time(fn, iters)
        ew = _hbm_roofline(16 * n, ms, peaks, src, "k_ew_fma_relu_scale_v4")
        ew.update(ms=ms)
        # 5 copies of X (320 MiB > L2): each timed call reads a copy the
        # previous four calls did not touch, so no L2 flush is needed.
        ncopy = 5
        Xs = [torch.randn(data.C2_X, device="cuda", generator=g) for _ in range(ncopy)]
        Xis = [torch.randint(-1000, 1001, data.C2_X, device="cuda", dtype=torch.int32,
                             generator=g) for _ in range(ncopy)]
        reds = {}
        for name, fn_, arrs in (("f32 sum last axis", lambda a: kernels.reduce_rows(a, REDUCE_SUM), Xs),
                                ("f32 max last axis", lambda a: kernels.reduce_rows(a, REDUCE_MAX), Xs),
                                ("f32 sum axis 0", lambda a: kernels.reduce_cols(a, REDUCE_SUM), Xs),
                                ("i32 sum last axis", lambda a: kernels.reduce_rows(a, REDUCE_SUM), Xis),
                                ("i32 max last axis", lambda a: kernels.reduce_rows(a, REDUCE_MAX), Xis)):
            it = iter(range(10 ** 9))
            f = lambda fn_=fn_, arrs=arrs: fn_(arrs[next(it) % ncopy])  # noqa: E731
            for _ in range(warm):
                f()
            rms = _graph_time(f, iters)
            r = _hbm_roofline(Xs[0].numel() * 4, rms, peaks, src, name)
            r.update(ms=rms, timing="CUDA graph of back-to-back launches")
            reds[name] = r
        line = {"metric": "config2 fused elementwise relu(a*b+c)*0.5 over 64M f32 (GB/s)",
                "value": ew["achieved"], "unit": "GB/s", "roofline": ew, "reductions": reds,
                "config": {"workload": "config2", "n": n, "X": list(data.C2_X),
                           "l2": "elementwise inputs 768 MiB > L2; reductions rotate over 5 "
                                 "copies of X (320 MiB > L2)",
                           "timing": "elementwise: back-to-back launches between CUDA events; "
                                     "reductions (~12 us each): a CUDA graph of back-to-back "
                                     "launches, so the host call rate does not bound them"}}
    elif config == "c3":
        nn_ = data.C3_N
        g = torch.Generator(device="cuda").manual_seed(8)
        A = (torch.rand((nn_, nn_), device="cuda", generator=g) * 2 - 1) / 64
        Bm = (torch.rand((nn_, nn_), device="cuda", generator=g) * 2 - 1) / 64
        G = torch.randn((nn_, nn_), device="cuda", generator=g) * 1e-2
        A_lo, B_lo, G_lo = kernels.split_lo(A), kernels.split_lo(Bm), kernels.split_lo(G)
        out = torch.empty((nn_, nn_), device="cuda")
        cases = {
            "C = A.B (K-major x MN-major)": lambda: kernels.gemm(A, Bm, a_lo=A_lo, b_lo=B_lo,
                                                                 b_mn_major=True, out=out),
            "dA = G.B^T (K-major x K-major)": lambda: kernels.gemm(G, Bm, a_lo=G_lo, b_lo=B_lo,
                                                                   out=out),
            "dB = A^T.G (MN-major x MN-major)": lambda: kernels.gemm(A, G, a_lo=A_lo, b_lo=G_lo,
                                                                     a_mn_major=True,
                                                                     b_mn_major=True, out=out),
        }
        flops = 2 * nn_ ** 3
        peak = peaks["bf16_tflops"] / 2 / 3
        res = {}
        for name, f in cases.items():
            for _ in range(warm):
                f()
            ms = _event_time(f, iters)
            tf = flops / (ms * 1e-3) / 1e12
            res[name] = {"ms": ms, "tflops": tf, "frac": tf / peak}
        avg = statistics.mean(r["tflops"] for r in res.values())
        line = {"metric": "config3 GEMM 4096^3 fp32 via 3xTF32 tcgen05 (algorithmic TFLOP/s)",
                "value": avg, "unit": "TFLOP/s",
                "roofline": {"bound": "tensor", "achieved": avg, "peak": peak, "unit": "TFLOP/s",
                             "frac": avg / peak, "traffic": None, "kernel": "k_gemm3x",
                             "peak_basis": f"{src} bf16_tflops (burst) / 2 (TF32) / 3 (3 MMAs)"},
                "contractions": res,
                "config": {"workload": "config3", "M": nn_, "N": nn_, "K": nn_,
                           "l2": "operands + residuals 256 MiB > L2"}}
    elif config == "c5gemm":
        # the three GEMM shapes of the config-5 step at one GPU, with the step's epilogues
        M, N = GLOBAL_BATCH, 4096
        g = torch.Generator(device="cuda").manual_seed(13)
        act = torch.rand((M, N), device="cuda", generator=g)
        W = torch.randn((N, N), device="cuda", generator=g) * (2.0 / N) ** 0.5
        Gm = torch.randn((M, N), device="cuda", generator=g) * 1e-4
        bias = torch.zeros(N, device="cuda")
        act_lo, W_lo, G_lo = kernels.split_lo(act), kernels.split_lo(W), kernels.split_lo(Gm)
        out, out_lo = torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")
        dW = torch.empty((N, N), device="cuda")
        from ferrograd_b200._lib import EPI_BIAS_RELU, EPI_RELU_MASK
        cases = {
            "forward act.W^T + b, relu (K x K)": (2 * M * N * N, lambda: kernels.gemm(
                act, W, a_lo=act_lo, b_lo=W_lo, epilogue=EPI_BIAS_RELU, bias=bias, out=out,
                out_lo=out_lo)),
            "dW = G^T.act (MN x MN)": (2 * M * N * N, lambda: kernels.gemm(
                Gm, act, a_lo=G_lo, b_lo=act_lo, a_mn_major=True, b_mn_major=True, out=dW)),
            "dX = mask(G.W) (K x MN)": (2 * M * N * N, lambda: kernels.gemm(
                Gm, W, a_lo=G_lo, b_lo=W_lo, b_mn_major=True, epilogue=EPI_RELU_MASK, mask=act,
                out=out, out_lo=out_lo)),
        }
        peak = peaks["bf16_tflops"] / 2 / 3
        res = {}
        for name, (fl, f) in cases.items():
            for _ in range(warm):
                f()
            ms = _event_time(f, iters)
            tf = fl / (ms * 1e-3) / 1e12
            res[name] = {"ms": ms, "tflops": tf, "frac": tf / peak}
        avg = statistics.mean(r["tflops"] for r in res.values())
        line = {"metric": "config5 GEMMs 8192x4096x4096 (3xTF32 tcgen05, algorithmic TFLOP/s)",
                "value": avg, "unit": "TFLOP/s",
                "roofline": {"bound": "tensor", "achieved": avg, "peak": peak, "unit": "TFLOP/s",
                             "frac": avg / peak, "traffic": None, "kernel": "k_gemm3x",
                             "peak_basis": f"{src} bf16_tflops (burst) / 2 (TF32) / 3 (3 MMAs)"},
                "contractions": res, "config": {"workload": "config5 GEMM shapes"}}
    elif config == "c4":
        Bx, C = data.C4
        g = torch.Generator(device="cuda").manual_seed(11)
        x = torch.randn((Bx, C), device="cuda", generator=g) * 2
        lab = torch.randint(0, C, (Bx,), device="cuda", generator=g)
        t = torch.nn.functional.one_hot(lab, C).float()
        fn = lambda: kernels.xent_fwd_bwd(x, t)  # noqa: E731
        for _ in range(warm):
            fn()
        ms = _event_time(fn, iters)
        r = _hbm_roofline(3 * Bx * C * 4, ms, peaks, src, "k_xent_rows_v4<8> + k_xent_loss_final")
        r.update(ms=ms)
        line = {"metric": "config4 cross-entropy fwd+bwd [65536,1000] f32 (GB/s)",
                "value": r["achieved"], "unit": "GB/s", "roofline": r,
                "config": {"workload": "config4", "shape": [Bx, C],
                           "l2": "logits + targets + dlogits 786 MB > L2"}}
    elif config in ("c1front", "c5front"):
        line = front_bench(config, iters, warm, peaks, src)
    elif config == "c2front":
        line = front_c2_bench(iters, warm, peaks, src)
    elif config == "c4front":
        line = front_c4_bench(iters, warm, peaks, src)
    else:
        raise SystemExit(f"unknown config {config}")
    del flush_buf
    return line


def front_bench(config, iters, warm, peaks, src):
    """The training step through the lazy-Tensor front end (the reference's
    public API: Linear / relu / cross_entropy / backward / Sgd::step /
    loss.to_vec(), examples/mnist.rs:90-97), every kernel scheduled, routed
    and launched per step."""
    import torch

    from ferrograd_b200 import data
    from ferrograd_b200 import front as F

    if config == "c1front":
        dims, B = (784, 128, 10), 256
    else:
        dims, B = (4096, 4096, 4096, 10), 8192
    x, t = data.mlp_batch(B, dims[0], dims[-1], 13, 14)
    F.reset_init_seed(42)
    model = F.Mlp(dims)
    opt = F.Sgd(model.parameters(), 0.01)
    xt, tt = F.tensor(x), F.tensor(t)
    for _ in range(warm):
        F.train_step(model, opt, xt, tt)
    F.synchronize()
    stream = torch.cuda.ExternalStream(F.stream())
    F.reset_stats()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    t0 = time.perf_counter()
    for _ in range(iters):
        loss = F.train_step(model, opt, xt, tt)
    wall_ms = (time.perf_counter() - t0) / iters * 1e3
    e1.record(stream)
    e1.synchronize()
    dev_ms = e0.elapsed_time(e1) / iters
    st = {k: v / iters for k, v in F.stats().items()}
    # End to end: the batch uploaded each step by Tensor::new from pinned host
    # memory (numpy views of page-locked torch tensors), the loss read back.
    xp = torch.from_numpy(x).pin_memory().numpy()
    tp = torch.from_numpy(t).pin_memory().numpy()
    t0 = time.perf_counter()
    for _ in range(iters):
        F.train_step(model, opt, F.tensor(xp), F.tensor(tp))
    e2e_ms = (time.perf_counter() - t0) / iters * 1e3
    nl = len(dims) - 1
    flops = sum(2 * B * dims[l] * dims[l + 1] * (3 if l > 0 else 2) for l in range(nl))
    return {"metric": f"config{'1' if dims[0] == 784 else '5'} MLP train steps/s through the "
                      "lazy-Tensor front end", "value": 1e3 / wall_ms, "unit": "steps/s",
            "roofline": _step_roofline(flops, dev_ms, peaks, src,
                                       "latency" if config == "c1front" else "tensor"),
            "flop_per_step": flops,
            "ms_per_step": wall_ms, "device_ms_per_step": dev_ms, "loss": loss,
            "per_step": st,
            "e2e": {"value": 1e3 / e2e_ms, "unit": "steps/s",
                    "h2d_bytes_per_step": int(x.nbytes + t.nbytes), "d2h_bytes_per_step": 4},
            "config": {"workload": config, "dims": list(dims), "batch": B,
                       "timing": "wall clock per step (loss.to_vec() synchronises each step); "
                                 "device time from CUDA events on the front end's stream"}}


def _front_time(fn, iters, stream):
    """Average device ms per fn() (which builds, schedules and realizes a
    Tensor graph) between CUDA events on the front end's stream."""
    import torch
    from ferrograd_b200 import front as F
    F.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def front_c2_bench(iters, warm, peaks, src):
    """Config 2 through the Tensor API (graph built, scheduled and launched
    per call): relu(a*b+c)*0.5 (one rendered 128-bit kernel), the row /
    column reductions of X (routed to the HBM reduction kernels), and two
    reductions of a lazy expression that the renderer maps to a warp per
    row and to a block per 32 columns."""
    import numpy as np
    import torch

    from ferrograd_b200 import data
    from ferrograd_b200 import front as F

    rng = np.random.default_rng(3)
    n = data.C2_N
    a, b, c = (F.tensor(rng.standard_normal(n, dtype=np.float32)) for _ in range(3))
    half = F.Tensor.scalar(0.5)
    for t in (a, b, c, half):
        t.realize()
    stream = torch.cuda.ExternalStream(F.stream())
    ew = lambda: a.mul(b).add(c).relu().mul(half).realize()  # noqa: E731
    for _ in range(warm):
        ew()
    F.reset_stats()
    ms = _front_time(ew, iters, stream)
    kernels_per_call = F.stats()["kernels"] / iters
    ew_r = _hbm_roofline(16 * n, ms, peaks, src, "rendered relu(a*b+c)*0.5 (float4)")
    ew_r.update(ms=ms, kernels_per_call=kernels_per_call)
    ncopy = 5  # 5 x 64 MiB > L2: each call reads a copy the previous four did not
    Xs = [F.tensor(rng.standard_normal(data.C2_X, dtype=np.float32)) for _ in range(ncopy)]
    Xis = [F.tensor(rng.integers(-1000, 1001, data.C2_X).astype(np.int32)) for _ in range(ncopy)]
    for t in Xs + Xis:
        t.realize()
    nbytes = int(np.prod(data.C2_X)) * 4
    reds = {}
    cases = (("f32 sum last axis (routed)", Xs, lambda x: x.sum([1]), 1),
             ("f32 max last axis (routed)", Xs, lambda x: x.max([1]), 1),
             ("f32 sum axis 0 (routed)", Xs, lambda x: x.sum([0]), 1),
             ("i32 sum last axis (routed)", Xis, lambda x: x.sum([1]), 1),
             ("i32 max last axis (routed)", Xis, lambda x: x.max([1]), 1),
             ("f32 sum last axis of x*x (rendered, warp per row)", Xs,
              lambda x: x.mul(x).sum([1]), 1),
             ("f32 sum axis 0 of x*x (rendered, block per 32 columns)", Xs,
              lambda x: x.mul(x).sum([0]), 1))
    for name, arrs, f, _ in cases:
        it = iter(range(10 ** 9))
        call = lambda f=f, arrs=arrs: f(arrs[next(it) % ncopy]).realize()  # noqa: E731
        for _ in range(warm):
            call()
        F.reset_stats()
        rms = _front_time(call, iters, stream)
        st = F.stats()
        r = _hbm_roofline(nbytes, rms, peaks, src, name)
        r.update(ms=rms, hand_reduce_per_call=st["hand_reduce"] / iters,
                 rendered_per_call=st["rendered"] / iters)
        reds[name] = r
    return {"metric": "config2 relu(a*b+c)*0.5 over 64M f32 through the Tensor API (GB/s)",
            "value": ew_r["achieved"], "unit": "GB/s", "roofline": ew_r, "reductions": reds,
            "config": {"workload": "c2front", "n": n, "X": list(data.C2_X),
                       "l2": "elementwise inputs 768 MiB > L2; reductions rotate over 5 copies "
                             "of X (320 MiB > L2)",
                       "timing": "CUDA events on the front end's stream around `steps` calls, "
                                 "each building, scheduling and launching its graph (host work "
                                 "included when it exceeds the kernel time)"}}


def front_c4_bench(iters, warm, peaks, src):
    """Config 4 through the Tensor API: logits.cross_entropy(targets), its
    gradient with respect to the logits, then the loss -- one fused
    fg_xent_fwd_bwd pass per call (the loss is taken from the gradient pass)."""
    import numpy as np
    import torch

    from ferrograd_b200 import data
    from ferrograd_b200 import front as F

    Bx, C = data.C4
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((Bx, C), dtype=np.float32) * 2).astype(np.float32)
    lab = rng.integers(0, C, Bx)
    t = np.zeros((Bx, C), np.float32)
    t[np.arange(Bx), lab] = 1.0
    lg = F.tensor(x).with_requires_grad(True)
    tt = F.tensor(t)
    lg.realize()
    tt.realize()

    def call():
        loss = lg.cross_entropy(tt)
        (g,) = loss.gradient([lg])
        g.realize()
        loss.realize()

    stream = torch.cuda.ExternalStream(F.stream())
    for _ in range(warm):
        call()
    F.reset_stats()
    ms = _front_time(call, iters, stream)
    st = {k: v / iters for k, v in F.stats().items() if k in ("kernels", "xent", "xent_reused")}
    r = _hbm_roofline(3 * Bx * C * 4, ms, peaks, src, "fg_xent_fwd_bwd via Tensor::cross_entropy")
    r.update(ms=ms)
    return {"metric": "config4 cross-entropy fwd+bwd [65536,1000] through the Tensor API (GB/s)",
            "value": r["achieved"], "unit": "GB/s", "roofline": r, "per_call": st,
            "config": {"workload": "c4front", "shape": [Bx, C],
                       "l2": "logits + targets + dlogits 786 MB > L2"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the configs 1-4 / front-end objects of the N=1 headline line")
    ap.add_argument("--dp", choices=["nccl", "peer"], default="nccl",
                    help="gradient exchange of the data-parallel step (N > 1)")
    ap.add_argument("--dp-chunks", type=int, default=4,
                    help="row chunks of layer 0's gradient in the peer-sharded exchange")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5", "c5gemm", "c1front",
                                         "c5front", "c2front", "c4front"], default="c5",
                    help="c5 (default) is the headline training step; c1-c4 time one config")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    if args.config != "c5":
        return config_bench(args)
    return our_arm(args)


if __name__ == "__main__":
    sys.exit(main())
