#!/usr/bin/env python3
"""Benchmark of the quantized-linear hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg4|cfg0|cfg1|cfg4_m8192]
                    [--exchange fused|multicast|gather] [--w4-packed-only]
    python bench.py --sweep [--sweep-cases cfg0,cfg1,...]   # every named shape, one GPU
    python bench.py --mlp [--mlp-rows M] [--gpus N]           # the cfg2 MLP block

Headline workload (default ``cfg4``): the W4A8 linear K=8192, N=28672 at M=512 tokens,
split column-parallel over N GPUs (each rank owns N/g output channels); every rank ends
with the whole fp16 [M][N] output.  The exchange: ``fused`` (default) -- the GEMM's
epilogues store each rank's columns into every rank's buffer over NVLink and a one-warp
peer-flag kernel signals completion; ``multicast`` -- the same with one store per element
through the NVSwitch multicast address of every rank's buffer; ``gather`` -- an NCCL
all-gather of the slabs and the [g][M][N/g] -> [M][N] assembly.  A step is one pass of the
path over one batch:
act-quant -> tcgen05 GEMM (-> exchange).  ``value`` is whole-job TOPS (2*M*K*N / step time,
device-timed with CUDA events, max over ranks), inputs resident in HBM, L2 flushed between
timed steps by a 256 MiB write outside the timed region.  Scaling is strong (the layer is
fixed).  Rank 0 compares the timed step's output with the C oracle (``parity``).

The line also carries: the decode half of the metric (W8A8 K=2560 N=9728 at M=1, GB/s,
weights rotated through 8 copies so they come from HBM; at N=1 also the same kernel on the
389 MB W8 lm_head 2560 -> 151936); the roofline of the dominant
kernel; the CPU baseline (the C oracle, a bounded row sample, all host threads and one
thread; rank 0, N=1); ``e2e`` through the reference-facing C-ABI call with host f32 buffers
(qlinear_run_f32 at N=1; H2D -> run with the exchange -> D2H at N>1); SM clocks sampled
during the timed region.

``--impl reference`` times the reference's CPU implementation of the path (the oracle
restatement of src/npu.rs:1097-1121 -- the reference's Rust crate cannot be built here)
on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# DRAM traffic of the dominant kernel per launch on the default workload
# (dram__bytes_read.sum + dram__bytes_write.sum = 246.04 MB + 18.01 MB) from the ncu capture
# summarised in profiles/gemm_w4a8_cfg4_m512.md (same workload, one GPU).
GEMM_TRAFFIC_BYTES = 264_049_408

WORKLOADS = {
    # name: (bits, K, N, M, description)
    "cfg4": (4, 8192, 28672, 512, "cfg4 W4A8 K8192 N28672 M512 split-N"),
    "cfg4_m8192": (4, 8192, 28672, 8192, "cfg4 W4A8 K8192 N28672 M8192 split-N"),
    "cfg0": (4, 2560, 9728, 512, "cfg0 W4A8 gate_proj K2560 N9728 M512"),
    "cfg1": (8, 2560, 9728, 1, "cfg1 W8A8 decode K2560 N9728 M1"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg4")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target CPU time of the oracle baseline sample")
    ap.add_argument("--exchange", choices=["gather", "fused", "multicast"], default="fused",
                    help="split-N output exchange at N>1: NCCL all-gather + column assembly, "
                         "or the kernels' epilogues storing into every rank's buffer")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle check of the timed step's output (profiling runs)")
    ap.add_argument("--sweep", action="store_true",
                    help="one GPU: one JSON line per named shape (cfg0-cfg4 and their M sweeps) "
                         "instead of the headline line")
    ap.add_argument("--sweep-cases", default="",
                    help="comma-separated case-name prefixes to run with --sweep (default all)")
    ap.add_argument("--swiglu-unfused", action="store_true",
                    help="prefill SwiGLU as GEMM -> f32 workspace -> SwiGLU pass (comparison)")
    ap.add_argument("--w4-packed-only", action="store_true",
                    help="W4 weights without their int8 copy (the prefill GEMM unpacks them)")
    ap.add_argument("--stream-k", action="store_true",
                    help="let the GEMM choose its stream-K schedule (QLINEAR_BACKEND_GEMM_STREAM_K)")
    ap.add_argument("--mlp", action="store_true",
                    help="time the cfg2 MLP block instead: one GPU qlinear_run_mlp_device, N GPUs "
                         "the split-K ShardedMLP")
    ap.add_argument("--mlp-rows", type=int, default=512)
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers
class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def int8_peak_tops(torch, dev) -> float:
    """Dense int8 tensor-core throughput of cuBLASLt on this GPU (torch._int_mm, 8192^3,
    best of 10 back-to-back launches): the int8 denominator MEASURED_PEAKS.json lacks."""
    a = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=dev).t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    del a, b
    return 2 * 8192 ** 3 / best / 1e12


def cpu_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return os.cpu_count(), model


def spread_rows(m_total, rows):
    """`rows` row indices spread evenly over [0, m_total): they cross every token tile and
    the last (tail) tiles of the GEMM's schedule, not only the first rows."""
    rows = max(1, min(int(rows), m_total))
    return np.unique(np.linspace(0, m_total - 1, rows).round().astype(np.int64))


def oracle_sample(bits, k, n, m_total, cpu_seconds, max_rows=None, threads=None, repeats=3):
    """Time the C oracle on a row sample sized to ~cpu_seconds per run (all host threads
    unless `threads` is given; the median of `repeats` runs).  The sample's rows are spread over the batch, and the oracle's
    output for them is returned, so that the caller can compare the timed GPU step with it.
    Returns (ops_per_s, row indices, seconds, threads, y f32 [rows][n])."""
    from oracle import oracle as O
    from open_rknpu2_lm_infer_b200 import workloads as W
    O.build()
    co = O.COracle()
    if threads is not None:
        co.set_threads(threads)
    threads = co.max_threads()
    w = W.weight_codes(bits, k, n)
    sw = W.weight_scales(n)
    x = W.activations(m_total, k)
    # probe with one row (warm), then size the sample
    co.linear(w, sw, x[:1])
    t0 = time.perf_counter()
    co.linear(w, sw, x[:1])
    t1 = time.perf_counter() - t0
    rows = int(max(1, min(m_total, cpu_seconds / max(t1, 1e-6))))
    if max_rows is not None:
        rows = min(rows, max_rows)
    idx = spread_rows(m_total, rows)
    xs = np.ascontiguousarray(x[idx])
    y, runs = None, []
    for _ in range(max(1, repeats)):
        t0 = time.perf_counter()
        out = co.linear(w, sw, xs)
        runs.append(time.perf_counter() - t0)
        y = out if y is None else y
    dt = statistics.median(runs)
    return 2.0 * len(idx) * k * n / dt, idx, dt, threads, y


def parity_record(y_gpu_rows, y_oracle, idx):
    """Bit-exact comparison of the GPU's fp16 rows with f16(oracle f32) (the oracle's f32
    value rounded once to nearest-even: the same single rounding the epilogue does)."""
    want = y_oracle.astype(np.float16)
    got = np.asarray(y_gpu_rows, dtype=np.float16)
    bad = got.view(np.uint16) != want.view(np.uint16)
    rec = {"rows_checked": int(len(idx)), "elements_checked": int(want.size),
           "mismatches": int(np.count_nonzero(bad)),
           "against": "f16(C oracle f32), bit-exact; rows spread over the batch",
           "rows": f"{int(idx[0])}..{int(idx[-1])} ({len(idx)} rows)"}
    if rec["mismatches"]:
        r, c = np.argwhere(bad)[0]
        rec["first_mismatch"] = {"row": int(idx[r]), "col": int(c),
                                 "got": float(got[r, c]), "want": float(want[r, c])}
    return rec


# ----------------------------------------------------------------------------- arms
def workload_config(args, world):
    """The `config` object of the JSON line; both arms print the same one."""
    bits, k, n, m, desc = WORKLOADS[args.workload]
    return {"workload": desc, "M": m, "K": k, "N": n, "bits": bits,
            "parallelism": f"split-N x{world}" + (
                "" if world == 1 else " + NCCL all-gather" if args.exchange == "gather" else
                " + output exchange fused into the kernels (NVLink)"),
            "l2": "flushed (256 MiB write) between timed steps, outside the timed region",
            "inputs": "fp16 N(0,1) with 1% x20 outlier channels, seed 42"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU implementation of the path (oracle port)."""
    if rank != 0:
        return
    bits, k, n, m, desc = WORKLOADS[args.workload]
    from oracle import oracle as O
    from open_rknpu2_lm_infer_b200 import workloads as W
    O.build()
    co = O.COracle()
    threads = co.max_threads()
    w = W.weight_codes(bits, k, n)
    sw = W.weight_scales(n)
    x = W.activations(m, k)
    co.linear(w, sw, x[:1])
    t0 = time.perf_counter()
    co.linear(w, sw, x[:1])
    t1 = time.perf_counter() - t0
    # each step: a bounded row sample so that warmup + steps stay within ~2 minutes
    budget = 100.0 / max(1, args.steps + args.warmup)
    rows = int(max(1, min(m, budget / max(t1, 1e-6))))
    for _ in range(args.warmup):
        co.linear(w, sw, x[:rows])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        co.linear(w, sw, x[:rows])
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    tops = 2.0 * rows * k * n / dt / 1e12
    cores, model = cpu_info()
    sample = (f"{rows} of {m} rows per step ({desc}), C oracle, {threads} OpenMP threads "
              f"(nproc {cores}), {model}")
    line = {
        "impl": "reference", "metric": "W4A8 linear TOPS (M=512) & decode GB/s (M=1), % of roofline, at 1/2/4/8 B200",
        "value": tops, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 * m / rows,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
    from open_rknpu2_lm_infer_b200 import workloads as W

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    bits, k, n, m, desc = WORKLOADS[args.workload]
    assert n % world == 0 and (n // world) % 8 == 0
    ns = n // world
    n0 = rank * ns

    backend = Backend(device=local_rank, w4_packed_only=args.w4_packed_only)
    codes = W.weight_codes(bits, k, n)
    scales = W.weight_scales(n)
    qm = QuantMatrix(bits, k, n, codes, scales)
    sharded = None
    fused = args.exchange in ("fused", "multicast")
    exchange_used = None
    if world > 1:
        # split-N; the [M][N] output put together on every rank either by an NCCL all-gather
        # of the slabs + column assembly, or (fused) by the kernels' epilogues storing each
        # rank's columns into every rank's buffer over NVLink
        from open_rknpu2_lm_infer_b200.sharded import ShardedLinear
        sharded = ShardedLinear(backend, qm, fused_exchange=fused, max_rows=m,
                                multicast=args.exchange == "multicast")
        exchange_used = {"fused": "fused into the kernels, NVLink peer stores "
                                  "(qlinear_run_device_scatter)",
                         "multicast": "fused into the kernels, NVSwitch multicast stores "
                                      "(qlinear_run_device_multicast)",
                         "gather": "NCCL all-gather + qlinear_interleave_columns"}[args.exchange]
        lin = sharded.linear
    else:
        lin = backend.load_shard(qm, n0, n0 + ns)
    del codes, qm
    backend.prepare(m)
    x_host = W.activations(m, k)
    x = torch.from_numpy(x_host).to(dev)
    y_local = torch.empty((m, ns), dtype=torch.float16, device=dev) if world == 1 else None
    y_full = torch.empty((m, n), dtype=torch.float16, device=dev) if world > 1 and not fused \
        else None
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def step():
        if world > 1 and fused:
            sharded.run_exchange(x, m, stream=stream)
        elif world > 1:
            sharded.run_device(x, y_full, m, stream=stream)
        else:
            lin.run_device(x, y_local, m, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()

    launches0 = backend.launches()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    backend.check(stream)

    # Clock record: nvidia-smi samples every 200 ms, longer than the timed region, so the
    # sampler also covers an untimed ~1 s soak of the same step right before it.
    # (the same step count on every rank: each step may hold a collective)
    t0 = time.perf_counter()
    for _ in range(4):
        step()
    torch.cuda.synchronize(dev)
    per_step = (time.perf_counter() - t0) / 4
    n_soak = torch.tensor([min(20000, int(1.0 / max(per_step, 1e-6)) + 1)], device=dev)
    if world > 1:
        dist.all_reduce(n_soak, op=dist.ReduceOp.MAX)
    soak_steps = int(n_soak.item())
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.25)
    for i in range(soak_steps):
        step()
        if i % 64 == 63:
            torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)

    def timed_steps():
        # Hold the GPU while the host enqueues every timed step, so the events measure
        # device time only (no host launch gaps inside a step).
        times = []
        torch.cuda._sleep(int(2e8))
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            times.append((e0, e1))
        torch.cuda.synchronize(dev)
        barrier()
        return times

    # The timed region: the steps as a caller runs them (no per-kernel events inside).
    launches_before = backend.launches()
    times = timed_steps()
    launches_timed = backend.launches() - launches_before
    clocks = sampler.stop()
    clocks["window"] = f"{soak_steps}-step untimed soak of the same step + the timed region"
    # The per-kernel breakdown (GEMM, act-quant) from the same number of steps run again with
    # the library's per-kernel events on; not part of `value`.
    backend.profile(True)
    timed_steps()
    backend.profile(False)
    quant_ms, main_ms, calls = backend.profile_collect()
    backend.check(stream)
    # the timed step's output, kept for the parity check against the oracle (rank 0)
    y_check = None
    if rank == 0 and not args.no_parity:
        src = y_local if world == 1 else (sharded.output[:m] if fused else y_full)
        y_check = src.cpu().numpy()
    step_s = sum(a.elapsed_time(b) for a, b in times) * 1e-3
    t = torch.tensor([step_s, main_ms * 1e-3, quant_ms * 1e-3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_s, main_s, quant_s = t.tolist()
    mean_step = step_s / args.steps
    ops = 2.0 * m * k * n
    value = ops / mean_step / 1e12

    # roofline of the dominant kernel (the GEMM on this rank's shard)
    per_launch = main_s / max(calls, 1)
    shard_ops = 2.0 * m * k * ns
    int8_peak = int8_peak_tops(torch, dev)
    achieved = shard_ops / per_launch / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                "frac": achieved / int8_peak,
                "peak_source": "int8 dense, measured by bench.py: cuBLASLt (torch._int_mm) "
                               "8192^3 burst; MEASURED_PEAKS.json has no int8 figure",
                "frac_of_nominal_4500": achieved / 4500.0,
                "traffic": GEMM_TRAFFIC_BYTES if (args.workload == "cfg4" and world == 1) else None,
                "traffic_source": "ncu dram bytes, profiles/gemm_w4a8_cfg4_m512.md",
                "kernel": "gemm_kernel (tcgen05.mma.cta_group::2 kind::i8, CTA pairs)",
                "kernel_ms": per_launch * 1e3, "act_quant_ms": quant_s / max(calls, 1) * 1e3}

    line = {
        "metric": "W4A8 linear TOPS (M=512) & decode GB/s (M=1), % of roofline, at 1/2/4/8 B200",
        "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_step * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": workload_config(args, world),
        "roofline": roofline,
        "exchange": exchange_used,
        "gpu_launches": int(launches_timed),
        "clocks": clocks,
    }
    # The split-N output exchange bounds the end-to-end scaling of this layer; report the
    # kernels' time beside the whole step.
    compute_s = (main_s + quant_s) / max(calls, 1)
    line["compute_only"] = {
        "value": ops / compute_s / 1e12, "unit": "TOPS", "per_step_us": compute_s * 1e6,
        "exchange_us": max(0.0, mean_step - compute_s) * 1e6,
        "note": "act-quant + GEMM device time per step (max over ranks; with the fused "
                "exchange the GEMM includes its peer stores), without the rest of the output "
                "exchange (all-gather + assembly, or the completion signal) that `value` "
                "includes"}

    # decode half of the metric: W8A8 K2560 N9728 M=1 (HBM-bound GEMV)
    if not args.no_decode:
        line["decode"] = decode_measure(backend, torch, dev, args, world)

    # end to end through the public C ABI with host buffers
    if not args.no_e2e:
        line["e2e"] = e2e_measure(backend, lin, torch, dist, dev, args, world, m, k, n, ns,
                                  x_host, sharded)

    line["gpu_launches"] = int(launches_timed)
    if sharded is not None:
        sharded.close()  # collective: unmaps the peers' buffers, frees this rank's
    else:
        lin.close()
    backend.close()
    if rank != 0:
        return
    # CPU legs after every collective of this arm (rank 0 only): the oracle's rows both time
    # the CPU baseline (N=1) and check the timed step's output
    cores, model = cpu_info()
    oracle_y = None
    if world == 1 and not args.no_cpu:
        ops_s, idx, dt, threads, oracle_y = oracle_sample(bits, k, n, m, args.cpu_seconds / 3)
        ops_1, idx1, dt1, _, _ = oracle_sample(bits, k, n, m, args.cpu_seconds / 4,
                                               threads=1, repeats=3)
        line["cpu_baseline"] = {
            "value": ops_s / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{len(idx)} of {m} rows of {desc} (spread over the batch): C oracle "
                      f"(oracle/qlinear_ref.c), OpenMP {threads} threads, median of 3 runs of "
                      f"{dt:.2f} s",
            "host": {"nproc": cores, "cpu_model": model},
            "single_thread": {"value": ops_1 / 1e12, "unit": "TOPS", "cores": 1,
                              "sample": f"{len(idx1)} of {m} rows, median of 3 runs of "
                                        f"{dt1:.2f} s"}}
    if y_check is not None:
        if oracle_y is None:
            _, idx, _, _, oracle_y = oracle_sample(bits, k, n, m, 6.0, max_rows=1024,
                                                   repeats=1)
        line["parity"] = parity_record(y_check[idx], oracle_y, idx)
    print(json.dumps(line), flush=True)


def decode_measure(backend, torch, dev, args, world):
    from open_rknpu2_lm_infer_b200 import QuantMatrix
    from open_rknpu2_lm_infer_b200 import workloads as W
    bits, k, n, m = 8, 2560, 9728, 1
    copies = 8  # 8 x 24.9 MB rotated: each call reads weights that are not in L2
    lins = []
    for c in range(copies):
        lins.append(backend.load(QuantMatrix(bits, k, n, W.weight_codes(bits, k, n, stream=c),
                                             W.weight_scales(n, stream=c))))
    x = torch.from_numpy(W.activations(m, k, stream=5)).to(dev)
    y = torch.empty((m, n), dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for i in range(3 * copies):
        lins[i % copies].run_device(x, y, m, stream=stream)
    torch.cuda.synchronize(dev)
    # A decode step runs its linears back to back, so the figure is the steady-state time of
    # one call (fused act-quant + GEMV) in a run of back-to-back calls, each reading a
    # different one of 8 weight copies (200 MB > L2: every call streams its weights from
    # HBM; no flush needed), one pair of CUDA events around 8 rotations.  Also reported:
    # one call alone, events around it (launch latency and the stream's ramp included).
    reps = 5
    per = 8 * copies
    runs = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(5e7))
        e0.record()
        for i in range(per):
            lins[i % copies].run_device(x, y, m, stream=stream)
        e1.record()
        torch.cuda.synchronize(dev)
        runs.append(e0.elapsed_time(e1) * 1e-3 / per)
    per_call = statistics.median(runs)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(per)]
    torch.cuda._sleep(int(2e8))
    for i in range(per):
        evs[i][0].record()
        lins[i % copies].run_device(x, y, m, stream=stream)
        evs[i][1].record()
    torch.cuda.synchronize(dev)
    backend.check(stream)
    alone = statistics.median(e0.elapsed_time(e1) * 1e-3 for e0, e1 in evs)
    wbytes = k * n * bits // 8 + 4 * n
    algo = wbytes + 2 * m * k + 2 * m * n
    hbm = measured_peaks().get("hbm_gbs", 6650.0)
    for l in lins:
        l.close()
    large = None
    if world == 1:
        # the largest decode linear of the cfg3 model, the W8 lm_head 2560 -> 151936 (389 MB):
        # the same kernel once a layer is long enough to amortise the per-launch ramp
        kl, nl = 2560, 151936
        codes_l, scales_l = W.weight_codes(8, kl, nl), W.weight_scales(nl)
        heads = [backend.load(QuantMatrix(8, kl, nl, codes_l, scales_l)) for _ in range(2)]
        del codes_l
        yl = torch.empty((1, nl), dtype=torch.float16, device=dev)
        xl = torch.from_numpy(W.activations(1, kl, stream=6)).to(dev)
        for i in range(4):
            heads[i % 2].run_device(xl, yl, 1, stream=stream)
        ts = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(int(5e7))
            e0.record()
            for i in range(8):
                heads[i % 2].run_device(xl, yl, 1, stream=stream)
            e1.record()
            torch.cuda.synchronize(dev)
            ts.append(e0.elapsed_time(e1) * 1e-3 / 8)
        backend.check(stream)
        tl = statistics.median(ts)
        bl = kl * nl + 4 * nl + 2 * kl + 2 * nl
        large = {"config": "lm_head W8A8 K2560 N151936 M1 (2 alternating copies, 778 MB)",
                 "call_us": tl * 1e6, "value": bl / tl / 1e9, "unit": "GB/s",
                 "frac": bl / tl / 1e9 / hbm}
        for h in heads:
            h.close()
    return {"large_layer": large,
            "config": "cfg1 W8A8 K2560 N9728 M1 (8 rotated weight copies, 200 MB > L2)",
            "call_us": per_call * 1e6,
            "call_us_alone": alone * 1e6,
            "value_alone": algo / alone / 1e9,
            "value": algo / per_call / 1e9, "unit": "GB/s",
            "roofline": {"bound": "hbm", "achieved": algo / per_call / 1e9, "peak": hbm,
                         "unit": "GB/s", "frac": algo / per_call / 1e9 / hbm,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)",
                         "timed": "steady-state call (fused act-quant + GEMV) in a run of "
                                  "back-to-back calls, CUDA events"}}


def e2e_measure(backend, lin, torch, dist, dev, args, world, m, k, n, ns, x_host, sharded):
    """Same metric through the public API with host buffers: H2D of the f32 input, the
    path (with the fused output exchange at N>1), D2H of the f32 output, every step;
    wall-clock between host synchronisations, max over ranks."""
    xin = np.ascontiguousarray(x_host.astype(np.float32))
    steps = max(3, min(args.steps, 10))
    pageable = None
    if world == 1:
        # the step's input and output in page-locked host memory (the library copies them by
        # DMA directly); the same call on ordinary pageable arrays is reported beside it
        def timed(x_arr, out_arr):
            for _ in range(2):
                lin.run(x_arr, out_arr, m)
            ts = []
            for _ in range(steps):
                t0 = time.perf_counter()
                lin.run(x_arr, out_arr, m)
                ts.append(time.perf_counter() - t0)
            return statistics.median(ts)
        pin_in = torch.from_numpy(xin).pin_memory()
        pin_out = torch.empty((m, n), dtype=torch.float32).pin_memory()
        dt = timed(pin_in.numpy(), pin_out.numpy())
        dt_pageable = timed(xin, np.empty((m, n), np.float32))
        pageable = {"value": 2.0 * m * k * n / dt_pageable / 1e12, "unit": "TOPS",
                    "ms_per_step": dt_pageable * 1e3,
                    "note": "the same call with ordinary (pageable) numpy buffers, which the "
                            "library stages through its pinned buffers"}
        h2d, d2h = m * k * 4, m * n * 4
    else:
        pin_in = torch.from_numpy(xin).pin_memory()
        pin_out = torch.empty((m, n), dtype=torch.float32).pin_memory()
        xd = torch.empty((m, k), dtype=torch.float32, device=dev)
        fused = args.exchange in ("fused", "multicast")
        if fused:
            sharded.add_exchange(m, torch.float32)  # the host API's type
        else:
            yf = torch.empty((m, n), dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream

        def one():
            xd.copy_(pin_in, non_blocking=True)
            if fused:
                y = sharded.run_exchange(xd, m, stream=stream, out_dtype=torch.float32)
            else:
                sharded.run_device(xd, yf, m, stream=stream)
                y = yf
            pin_out.copy_(y, non_blocking=True)
            torch.cuda.synchronize(dev)
        for _ in range(2):
            one()
        ts = []
        for _ in range(steps):
            dist.barrier()
            t0 = time.perf_counter()
            one()
            ts.append(time.perf_counter() - t0)
        dt = statistics.median(ts)
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = t.item()
        h2d, d2h = m * k * 4, m * n * 4
    return {"value": 2.0 * m * k * n / dt / 1e12, "unit": "TOPS", "ms_per_step": dt * 1e3,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "host_buffers": "page-locked", "pageable": pageable,
            "api": "qlinear_run_f32 (host f32 in/out)" if world == 1 else
                   "H2D f32 -> qlinear_run_device_scatter (fused NVLink output exchange) -> "
                   "D2H f32" if args.exchange == "fused" else
                   "H2D f32 -> qlinear_run_device_multicast (NVSwitch multicast output "
                   "exchange) -> D2H f32" if args.exchange == "multicast" else
                   "H2D f32 -> qlinear_run_device -> NCCL all-gather -> "
                   "qlinear_interleave_columns -> D2H f32"}


def run_mlp(args, rank, world, local_rank):
    """--mlp: the cfg2 MLP block (W4 gate/up 2560 -> 2 x 9728 + SwiGLU -> f32 middle -> W8
    down 9728 -> 2560) at --mlp-rows tokens.  One GPU: qlinear_run_mlp_device; N GPUs: the
    split-K ShardedMLP (gate/up columns and down rows split together, NCCL all-reduces of the
    row maxima and the int32 partial accumulators).  TOPS of the whole block; device time per
    step with CUDA events (GPU held while the host enqueues; L2 flushed between steps outside
    the timed region), max over ranks.  Strong scaling."""
    import torch
    import torch.distributed as dist
    from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
    from open_rknpu2_lm_infer_b200 import workloads as W
    from open_rknpu2_lm_infer_b200.sharded import ShardedMLP
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hidden, h, m = 2560, 9728, args.mlp_rows
    gate_up = QuantMatrix(4, hidden, 2 * h, W.weight_codes(4, hidden, 2 * h, stream=90),
                          W.weight_scales(2 * h, stream=90))
    down = QuantMatrix(8, h, hidden, W.weight_codes(8, h, hidden, stream=91),
                       W.weight_scales(hidden, stream=91))
    backend = Backend(device=local_rank, w4_packed_only=args.w4_packed_only)
    x = torch.from_numpy(W.activations(m, hidden, stream=92)).to(dev)
    y = torch.empty((m, hidden), dtype=torch.float16, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if world > 1:
        mlp = ShardedMLP(backend, gate_up, down)
        step = lambda: mlp.run_device(x, y, m, stream=stream)  # noqa: E731
    else:
        gu, dn = backend.load(gate_up), backend.load(down)
        step = lambda: backend.run_mlp_device(gu, dn, x, y, m, stream=stream)  # noqa: E731
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ev = []
    torch.cuda._sleep(int(2e8))
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        ev.append((e0, e1))
    torch.cuda.synchronize(dev)
    backend.check(stream)
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in ev) * 1e-3 / args.steps],
                     dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    per = t.item()
    ops = 2.0 * m * hidden * 2 * h + 2.0 * m * h * hidden
    if rank == 0:
        print(json.dumps({
            "metric": "cfg2 MLP block TOPS (W4 gate/up + SwiGLU, W8 down)", "value": ops / per / 1e12,
            "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "strong",
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"cfg2 MLP block M={m}", "M": m, "hidden": hidden,
                       "intermediate": h,
                       "parallelism": "one GPU" if world == 1 else
                       f"split-K x{world} (gate/up columns + down rows, all-reduce of row "
                       "maxima and int32 accumulators)",
                       "l2": "flushed between timed steps, outside the timed region"}}),
            flush=True)
    if world > 1:
        mlp.close()
    backend.close()


def run_sweep(args):
    """--sweep: every named shape on one GPU, one JSON line each.

    Every case runs its calls back to back (the way a model runs its linears) over enough
    distinct weight copies that each call streams its weights from HBM (a rotation larger
    than the L2 cache, or one layer set larger than it); activations are re-used and may sit
    in L2.  Time = CUDA events around a whole rotation, the GPU held by a sleep kernel while
    the host enqueues, median of 5.  TOPS = 2*M*K*N (summed over the case's linears) / time;
    GB/s = the case's algorithmic bytes (weights as stored for the kernel that reads them,
    scales, fp16 activations in and out) / time.
    """
    import torch
    from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
    from open_rknpu2_lm_infer_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    backend = Backend(device=0, swiglu_unfused=args.swiglu_unfused, gemm_stream_k=args.stream_k,
                      w4_packed_only=args.w4_packed_only)
    stream = torch.cuda.current_stream(dev).cuda_stream
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    hbm = measured_peaks().get("hbm_gbs", 6650.0)
    int8_peak = int8_peak_tops(torch, dev)
    only = [s for s in args.sweep_cases.split(",") if s]
    codes_cache = {}

    def load(bits, k, n, copies):
        key = (bits, k, n)
        if key not in codes_cache:
            codes_cache[key] = (W.weight_codes(bits, k, n), W.weight_scales(n))
        c, s = codes_cache[key]
        return [backend.load(QuantMatrix(bits, k, n, c, s)) for _ in range(copies)]

    def act(m, k, stream_id=0):
        return torch.from_numpy(W.activations(m, k, stream=stream_id)).to(dev)

    def time_chain(chain, reps=5):
        """chain(): enqueue one rotation; returns seconds per rotation (median)."""
        chain()
        chain()
        torch.cuda.synchronize(dev)
        runs = []
        for _ in range(reps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(int(5e7))
            e0.record()
            chain()
            e1.record()
            torch.cuda.synchronize(dev)
            runs.append(e0.elapsed_time(e1) * 1e-3)
        backend.check(stream)
        return statistics.median(runs)

    def copies_for(bytes_per_copy):
        return max(2, min(16, -(-4 * l2 // max(1, bytes_per_copy))))

    def kernel_bytes(bits, k, n, m):
        """Weight bytes the path's kernel reads: the packed W4 copy, except for a W4
        prefill GEMM of a backend that keeps the int8 expansion (it reads that)."""
        w4_int8 = m > 8 and backend.stats().get("w4_prefill") == "int8 copy"
        wb = k * n * (bits // 8 if bits == 8 else (1 if w4_int8 else 0.5))
        return int(wb) + 4 * n

    def emit(case, m, secs, ops, bytes_, launches, extra=None):
        line = {"sweep": case, "M": m, "us": secs * 1e6, "tops": ops / secs / 1e12,
                "gbs": bytes_ / secs / 1e9,
                "frac_int8_peak": ops / secs / 1e12 / int8_peak,
                "frac_hbm": bytes_ / secs / 1e9 / hbm,
                "bound": "hbm" if m <= 16 else "tensor",
                "launches": launches}
        if extra:
            line.update(extra)
        print(json.dumps(line), flush=True)

    def want(name):
        return not only or any(name.startswith(p) for p in only)

    sampler = ClockSampler(0)
    sampler.start()
    launches0 = backend.launches()

    # single linears: cfg0 (W4A8 M512), cfg1 (W8A8 M1, M4), cfg4 (W4A8 M 1/8/512/8192)
    singles = [("cfg0", 4, 2560, 9728, (512,)), ("cfg1", 8, 2560, 9728, (1, 4)),
               ("cfg4", 4, 8192, 28672, (1, 8, 512, 8192))]
    for name, bits, k, n, ms in singles:
        if not want(name):
            continue
        ncopy = copies_for(kernel_bytes(bits, k, n, max(ms)))
        lins = load(bits, k, n, ncopy)
        for m in ms:
            x = act(m, k)
            y = torch.empty((m, n), dtype=torch.float16, device=dev)
            reps = max(1, min(8, int(2e11 / (2.0 * m * k * n * ncopy)) + 1))

            def chain():
                for _ in range(reps):
                    for lin in lins:
                        lin.run_device(x, y, m, stream=stream)
            b0 = backend.launches()
            secs = time_chain(chain) / (reps * ncopy)
            launches = (backend.launches() - b0) / (7 * reps * ncopy)
            emit(f"{name} W{bits}A8 K{k} N{n}", m, secs, 2.0 * m * k * n,
                 kernel_bytes(bits, k, n, m) + 2 * m * k + 2 * m * n, launches,
                 {"copies": ncopy})
            del x, y
        for lin in lins:
            lin.close()
        del lins
        codes_cache.clear()

    # cfg2: MLP block gate/up W4 (2560 -> 2x9728, SwiGLU in the epilogue) -> down W8
    if want("cfg2"):
        k, h = 2560, 9728
        blk_bytes = kernel_bytes(4, k, 2 * h, 512) + kernel_bytes(8, h, k, 512)
        ncopy = copies_for(blk_bytes)
        gus = load(4, k, 2 * h, ncopy)
        downs = load(8, h, k, ncopy)
        for m in (1, 16, 128, 512, 4096):
            x = act(m, k)
            y = torch.empty((m, k), dtype=torch.float16, device=dev)

            def chain():
                for gu, dn in zip(gus, downs):
                    backend.run_mlp_device(gu, dn, x, y, m, stream=stream)
            b0 = backend.launches()
            secs = time_chain(chain) / ncopy
            launches = (backend.launches() - b0) / (7 * ncopy)
            ops = 2.0 * m * k * 2 * h + 2.0 * m * h * k
            bytes_ = (kernel_bytes(4, k, 2 * h, m) + kernel_bytes(8, h, k, m)
                      + 2 * m * k + 2 * m * h + 2 * m * h + 2 * m * k)
            emit("cfg2 MLP block W4 gate/up+SwiGLU -> W8 down (qlinear_run_mlp_device)", m, secs,
                 ops, bytes_, launches,
                 {"copies": ncopy})
        for lin in gus + downs:
            lin.close()
        del gus, downs
        codes_cache.clear()

    # cfg3: the linears of 36 decoder layers (W4/W8 per linear from the seeded draw), loaded
    # and called through DenseLayerLinears the way the reference's dense model does it
    if want("cfg3"):
        from open_rknpu2_lm_infer_b200.layers import DenseLayerLinears
        Q = W.QWEN3_4B
        mbits = W.cfg3_module_bits(Q["layers"])
        ck = W.SyntheticCheckpoint(mbits, share_by_shape=True)
        layers = [DenseLayerLinears.load(backend, ck, f"model.layers.{i}.", Q["hidden"],
                                         Q["q_heads"], Q["kv_heads"], Q["head_dim"],
                                         Q["intermediate"]) for i in range(Q["layers"])]
        n_w4 = sum(lin.bits == 4 for layer in layers for _, lin, _ in layer.linears())
        n_lin = sum(1 for layer in layers for _ in layer.linears())
        for m in (1, 512):
            xs = {k: act(m, k, stream_id=k) for k in (2560, 4096)}
            outs = {n: torch.empty((m, n), dtype=torch.float16, device=dev) for n in (6144, 2560)}

            def chain():
                for layer in layers:
                    layer.qkv_device(xs[2560], outs[6144], m, stream=stream)
                    layer.o_device(xs[4096], outs[2560], m, stream=stream)
                    # the MLP: gate/up + SwiGLU -> f32 middle -> down
                    layer.mlp_device(xs[2560], outs[2560], m, stream=stream)
            b0 = backend.launches()
            secs = time_chain(chain, reps=3)
            launches = (backend.launches() - b0) / 5
            ops = bytes_ = 0.0
            for layer in layers:
                for role, lin, _ in layer.linears():
                    k, n = lin.k(), lin.n()
                    ops += 2.0 * m * k * n
                    bytes_ += kernel_bytes(lin.bits, k, n, m) + 2 * m * k + 2 * m * (
                        n // 2 if role == "gate_up" else n)
            emit(f"cfg3 36 layers x (qkv, o, gate/up+SwiGLU, down) through DenseLayerLinears, "
                 f"{n_w4}/{n_lin} linears W4", m, secs, ops, bytes_, launches,
                 {"ms_per_pass": secs * 1e3})
            if m == 1:
                # the same decode pass captured once into a CUDA graph and replayed (every
                # call at one token allocates nothing; the launches' programmatic stream
                # serialization becomes programmatic edges of the graph)
                g = torch.cuda.CUDAGraph()
                cap = torch.cuda.Stream(dev)
                cap.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(cap):
                    stream_saved = stream
                    stream = cap.cuda_stream
                    chain()  # warm on the capture stream
                    cap.synchronize()
                    with torch.cuda.graph(g, stream=cap):
                        chain()
                    stream = stream_saved
                torch.cuda.current_stream(dev).wait_stream(cap)
                secs_g = time_chain(g.replay, reps=3)
                emit(f"cfg3 36 layers decode pass as one CUDA graph (replay)", m, secs_g, ops,
                     bytes_, launches, {"ms_per_pass": secs_g * 1e3})
                del g
        for layer in layers:
            layer.close()

    # lm_head: W8 2560 -> 151936 (the vocabulary projection of the Qwen3-4B-shaped model)
    if want("lmhead"):
        from open_rknpu2_lm_infer_b200.layers import OutputHead
        bits, k, n = 8, 2560, 151936
        ckh = W.SyntheticCheckpoint({"lm_head": 8})
        # 2 x 389 MB: every call streams from HBM
        heads = [OutputHead.quantized(backend, ckh, n, k) for _ in range(2)]
        lins = [h.linear for h in heads]
        for m in (1, 512):
            x = act(m, k)
            y = torch.empty((m, n), dtype=torch.float16, device=dev)

            def chain():
                for head in heads:
                    head.run_device(x, y, m, stream=stream)
            b0 = backend.launches()
            secs = time_chain(chain) / len(lins)
            launches = (backend.launches() - b0) / (7 * len(lins))
            emit(f"lmhead W8A8 K{k} N{n} (OutputHead)", m, secs, 2.0 * m * k * n,
                 kernel_bytes(bits, k, n, m) + 2 * m * k + 2 * m * n, launches, {"copies": 2})
            del x, y
        for head in heads:
            head.close()
        codes_cache.clear()

    clocks = sampler.stop()
    print(json.dumps({"sweep_done": True, "swiglu": "unfused" if args.swiglu_unfused else
                      "fused in the GEMM epilogue (prefill)", "stream_k": args.stream_k,
                      "int8_peak_tops": int8_peak,
                      "hbm_gbs": hbm,
                      "l2_bytes": l2, "clocks": clocks,
                      "launches_total": backend.launches() - launches0}), flush=True)
    backend.close()


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world > 1:
        print(f"--gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.sweep:
        if world == 1:
            run_sweep(args)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.mlp:
            run_mlp(args, rank, world, local_rank)
            return
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
