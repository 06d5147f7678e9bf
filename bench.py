#!/usr/bin/env python
"""Benchmark of the jax-rs B200 backend's hot path.

Default workload (the headline): f32 GEMM M=N=K=8192 through the C ABI
(jx_gemm_f32, tcgen05 3xTF32), one GEMM per step.  With --gpus N each rank
computes its own 8192-row shard of a (8192*N) x 8192 x 8192 product with a
replica of B (M-row sharding, no collective), so per-GPU work is fixed: weak
scaling (--strong splits the rows of one --size^3 product instead).  The
default line also carries `wide_mlp`: data-parallel training of the wide MLP
(8192 -> 4 x 8192 GELU -> 1000, global batch 65536 split over the N ranks,
NCCL gradient all-reduce per layer), timed in the same process.  Other
workloads (--workload): chain, chain_grad, rng, rowsum, argmax, fullsum,
sum_vjp, max_vjp, bgemm, conv, fft1d, fft2d (these four split their global
batch over the ranks), mlp, wide_mlp, conv1d, pool, batchnorm.

Timing: W warm-up steps, then exactly K steps between barrier +
torch.cuda.synchronize(), CUDA events on the launching stream, max over
ranks.  Operands are 256 MiB each (larger than the 126 MB L2).

`--impl reference` times the reference's CPU implementation of the same
workload (the oracle's C restatement of jax-rs's CPU loop on one host
thread, as the single-threaded reference runs, a bounded row sample per
step) and prints the same JSON line.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib
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

METRIC = "f32 GEMM TFLOP/s + MLP train samples/s at 1/2/4/8 B200; fused-elt HBM GB/s"


WORKLOADS = ("sgemm", "chain", "chain_grad", "rng", "rowsum", "argmax", "fullsum", "mlp", "wide_mlp", "fft1d",
             "fft2d", "conv", "bgemm", "conv1d", "pool", "batchnorm", "sum_vjp", "max_vjp")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="sgemm",
                   help="one of " + ", ".join(WORKLOADS) + "; a comma-separated list runs each in turn in the "
                        "same processes and prints one line per workload")
    p.add_argument("--precision", default=None, choices=["3xtf32", "exact"],
                   help="GEMM precision of the MLP trainer (default: exact for mlp, whose one-tile products the "
                        "sequential-k kernel runs faster and bit-identically; 3xtf32 for wide_mlp)")
    p.add_argument("--global-batch", type=int, default=65536, help="wide MLP global batch")
    p.add_argument("--fft-batch", type=int, default=0, help="override the FFT batch (smaller cases for profiling)")
    p.add_argument("--conv-batch", type=int, default=0, help="override the conv batch (smaller cases for profiling)")
    p.add_argument("--conv-kernel", default="auto", choices=["auto", "one_cta", "pair"],
                   help="implicit conv kernel (jx_conv_set_kernel); auto picks the SM-pair kernel at the default size")
    p.add_argument("--size", type=int, default=8192, help="GEMM M=N=K per rank (with --strong: of the whole product)")
    p.add_argument("--gemm-prec", default="3xtf32", choices=["3xtf32", "pair"],
                   help="sgemm/bgemm: JX_PREC_3XTF32 (the dispatcher's choice) or JX_PREC_3XTF32_PAIR (SM-pair "
                        "kernel, split in shared memory)")
    p.add_argument("--strong", action="store_true",
                   help="sgemm: split the M rows of one size^3 product over the ranks (strong scaling) instead of "
                        "giving every rank its own size-row shard")
    p.add_argument("--no-wide-mlp", action="store_true",
                   help="sgemm: skip the wide-MLP data-parallel measurement the default line carries")
    p.add_argument("--wide-steps", type=int, default=8, help="timed steps of that wide-MLP measurement")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-rows", type=int, default=8, help="GEMM rows timed by the CPU baseline")
    args = p.parse_args()
    for wl in args.workload.split(","):
        if wl not in WORKLOADS:
            p.error(f"unknown workload {wl!r}")
    return args


# DRAM bytes (read + write) per launch of each workload's dominant kernel at
# the default size, from one ncu capture of dram__bytes_read.sum +
# dram__bytes_write.sum, taken once, not in this run.  FFT and conv were
# captured on a smaller batch and scaled by the batch; their traffic is
# proportional to it.  batchnorm sums its three kernels (the roofline covers
# the whole call).  None for any other size.
TRAFFIC = {
    "sgemm": 3.1289e9 + 0.2588e9,            # gemm_pair_kernel<0,1>, 8192^3
    "chain": 1.0738e9 + 1.0275e9,            # jx_tape_kernel, 2^28
    "rowsum": 1.0738e9 + 0.0039e9,           # reduce_rows_kernel<sum>
    "argmax": 1.0738e9 + 0.0033e9,           # argreduce_rows_kernel<max>
    "fullsum": 1.0738e9 + 0.0049e9,          # reduce_all_pass1<sum>
    "fft1d": 4 * (0.5369e9 + 0.4847e9),      # fft_kernel<12>, batch 16384 x 4
    "fft2d": 8 * (0.2685e9 + 0.2158e9),      # column pass fft1024_tma_kernel, batch 32 x 8
    "conv": 4 * (0.0563e9 + 0.0067e9 + 0.0563e9 + 0.0032e9 + 0.1549e9 + 0.0006e9),  # 3 conv_pair_kernel, B 16 x 4
    "bgemm": 3.4474e9 + 1.0573e9,            # gemm_pair_kernel<0,1>, [64,2048,2048]^2
    "pool": 0.8228e9 + 0.1918e9,             # pool2d_kernel<max,3,3>, [64,256,112,112]
    "batchnorm": (0.2055e9 + 0.0036e9) + 0.0005e9 + (0.2056e9 + 0.1571e9),  # stats + finalize + apply
    "conv1d": 0.2704e9 + 0.2296e9,           # conv1d_kernel<1,3>, [64,256,4096]
    "sum_vjp": 0.0003e9 + 1.0131e9,          # sum_rows_vjp_kernel, [65536,4096]
    "max_vjp": 1.0742e9 + 1.0265e9,          # max_rows_vjp_reg_kernel<4>, [65536,4096]
    "rng": 0.0043e9 + 1.0194e9,              # rng_kernel, 2^28 draws
    "mlp": 0.0033e9 + 0.0,                   # mlp_fused_step_kernel, batch 128 (weights stay in L2)
}


TRAFFIC_BASIS = "ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of the default size, not this run"
BATCH_SPLIT = ("fft1d", "fft2d", "conv", "bgemm")  # workloads whose global batch splits over the ranks


def traffic_for(args, world=1):
    """Per-launch DRAM bytes of this rank's dominant kernel, or None.  Where
    the global batch splits over the ranks, a rank's launch moves its share."""
    default = (args.size == 8192 and not args.fft_batch and not args.conv_batch and not args.strong)
    if args.workload == "mlp" and args.precision not in (None, "exact"):
        return None  # the figure is the fused exact step's
    t = TRAFFIC.get(args.workload) if default else None
    if t is not None and args.workload in BATCH_SPLIT:
        t /= world
    elif t is not None and world > 1 and args.workload != "sgemm":
        return None
    return t


def load_peaks(clocks=None, timed_ms=0.0):
    """(HBM GB/s, bf16 TFLOP/s, basis).  The bf16 figure is the burst one
    (the profiling recipe's denominator for a kernel timed on its own), or
    the sustained one when the timed region ran for a second or more with
    the power cap active and the SM clock held below 90% of its maximum: a
    loop like that settles at the capped clock the sustained figure was
    measured at.  (The cap flag alone is not enough: runs at full clock
    report it too.)"""
    c = clocks or {}
    slow = bool(c.get("sm_mhz")) and bool(c.get("sm_max_mhz")) and c["sm_mhz"] < 0.9 * c["sm_max_mhz"]
    capped = "sw_power_cap" in (c.get("reasons") or []) and slow and timed_ms >= 1000.0
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        if capped and "bf16_tflops_sustained" in pk:
            return float(pk["hbm_gbs"]), float(pk["bf16_tflops_sustained"]), "measured sustained (power cap active)"
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, (1400.0 if capped else 1590.0), "fallback"


def at_run_clock(achieved, clocks):
    """achieved / (the burst 3xTF32 peak scaled by the timed region's median
    SM clock over the maximum SM clock), or None without clock samples: how
    close a tensor-bound kernel came to the peak at the clock it actually ran
    at (a power-capped box runs below the clock the peak was measured at)."""
    mhz, mx = (clocks or {}).get("sm_mhz"), (clocks or {}).get("sm_max_mhz")
    if not mhz or not mx:
        return None
    _, bf16, _ = load_peaks()
    return round(achieved / (bf16 / 6.0 * float(mhz) / float(mx)), 4)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        # a short timed region ends before the first 100 ms sample: wait (up
        # to 1 s) for two samples so the line always carries a clock reading
        t0 = time.time()
        while len(self.lines) < 2 and time.time() - t0 < 1.0:
            time.sleep(0.05)
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


class Dist:
    def __init__(self, n):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v):
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


def shard(global_n, dist, what):
    """This rank's share of a global count that splits evenly over the ranks."""
    if global_n % dist.world:
        raise SystemExit(f"{what} {global_n} does not split evenly over {dist.world} ranks")
    return global_n // dist.world


# ---------------------------------------------------------------------------
# CPU reference (oracle) timing -- the only place bench.py runs oracle code
# ---------------------------------------------------------------------------
def _split_run(fn, parts, threads):
    """Run fn over parts on `threads` host threads (the oracle's C calls
    release the GIL)."""
    if threads <= 1 or len(parts) <= 1:
        return [fn(p) for p in parts]
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(threads) as ex:
        return list(ex.map(fn, parts))


def cpu_measure(args, threads, budget_s=8.0):
    """The reference's CPU path (the oracle's restatement, same loop order) on
    a bounded sample of the workload, repeated until about budget_s seconds.
    Returns (value, unit, seconds per repetition, sample description)."""
    import oracle as O
    O.build()
    wl = args.workload
    rng = np.random.default_rng(7)
    par = f"{threads} host thread{'s' if threads > 1 else ''}"
    if wl == "sgemm":
        rows = args.cpu_rows
        a = rng.uniform(-1, 1, (rows, args.size)).astype(np.float32)
        b = rng.uniform(-1, 1, (args.size, args.size)).astype(np.float32)
        fn, work, unit = (lambda: O.matmul(a, b, nthreads=threads)), 2.0 * rows * args.size ** 2 / 1e12, "TFLOP/s"
        sample = f"{rows} rows of the {args.size}^3 product"
    elif wl == "bgemm":
        rows, n = 64, 2048
        a = rng.uniform(-1, 1, (rows, n)).astype(np.float32)
        b = rng.uniform(-1, 1, (n, n)).astype(np.float32)
        fn, work, unit = (lambda: O.matmul(a, b, nthreads=threads)), 2.0 * rows * n * n / 1e12, "TFLOP/s"
        sample = f"{rows} rows of one [2048,2048] x [2048,2048] batch entry"
    elif wl == "chain":
        n = 1 << 22
        x = rng.standard_normal(n).astype(np.float32)
        parts = np.array_split(x, max(1, threads))
        fn = lambda: _split_run(lambda p: O.chain_fwd(p, np.float32(1.1), np.float32(0.9)), parts, threads)
        work, unit, sample = 8.0 * n / 1e9, "GB/s", f"2^22 elements of the 2^28 chain"
    elif wl == "rng":
        n = 1 << 24
        k = O.key_from_seed(1).split()[0]
        fn = lambda: O.uniform_range(k, n, -1.0, 1.0)
        work, unit, sample = 4.0 * n / 1e9, "GB/s", "2^24 of the 2^28 draws (the stream is sequential: 1 thread)"
    elif wl == "chain_grad":
        n = 1 << 22
        x = rng.standard_normal(n).astype(np.float32)
        parts = np.array_split(x, max(1, threads))
        fn = lambda: _split_run(lambda p: O.chain_vjp(p, np.float32(1.1), np.float32(0.9)), parts, threads)
        work, unit, sample = 12.0 * n / 1e9, "GB/s", f"2^22 elements of the 2^28 chain, value and gradient"
    elif wl in ("rowsum", "argmax"):
        x = rng.standard_normal((4096, 4096)).astype(np.float32)
        if wl == "rowsum":
            fn = lambda: O.reduce_axis(x, 1, "sum", nthreads=threads)
        else:
            fn = lambda: O.arg_rows(x, True, nthreads=threads)
        work, unit, sample = (4.0 * x.size + 4.0 * 4096) / 1e9, "GB/s", "4096 of the 65536 rows"
    elif wl in ("sum_vjp", "max_vjp"):
        x = rng.standard_normal((4096, 4096)).astype(np.float32)
        ct = rng.standard_normal(4096).astype(np.float32)
        if wl == "sum_vjp":
            fn = lambda: O.sum_rows_vjp(ct, 4096)
            work = (4.0 * 4096 + 4.0 * x.size) / 1e9
        else:
            fn = lambda: O.max_rows_vjp(x, ct)
            work = (8.0 * x.size + 4.0 * 4096) / 1e9
        unit, sample = "GB/s", "4096 of the 65536 rows (1 thread)"
    elif wl == "fullsum":
        n = 1 << 24
        x = rng.standard_normal(n).astype(np.float32)
        parts = np.array_split(x, max(1, threads))
        fn = lambda: _split_run(lambda p: O.reduce_all(p, "sum"), parts, threads)
        work, unit, sample = 4.0 * n / 1e9, "GB/s", "2^24 of the 2^28 elements"
    elif wl == "fft1d":
        x = rng.standard_normal((256, 4096, 2)).astype(np.float32)
        fn = lambda: O.fft_c2c(x, nthreads=threads)
        work, unit, sample = 16.0 * 256 * 4096 / 1e9, "GB/s", "256 of the 65536 transforms"
    elif wl == "fft2d":
        x = rng.standard_normal((2, 1024, 1024, 2)).astype(np.float32)
        fn = lambda: O.fft2_c2c(x, nthreads=threads)
        work, unit, sample = 16.0 * 2 * 1024 * 1024 / 1e9, "GB/s", "2 of the 256 images"
    elif wl == "conv":
        C = O_ = 256
        x = rng.standard_normal((1, C, 56, 56)).astype(np.float32)
        w = (rng.standard_normal((O_, C, 3, 3)) * np.sqrt(2.0 / (C * 9))).astype(np.float32)
        g = rng.standard_normal((1, O_, 56, 56)).astype(np.float32)

        def fn():
            O.conv2d_fwd(x, w, 1, 1, nthreads=threads)
            O.conv2d_bwd_data(g, w, x.shape, 1, 1, nthreads=threads)
            O.conv2d_bwd_filter(x, g, w.shape, 1, 1, nthreads=threads)
        work, unit, sample = 3 * 2.0 * O_ * C * 9 * 56 * 56 / 1e12, "TFLOP/s", "1 of the 64 images, forward + dX + dW"
    elif wl == "conv1d":
        x = rng.standard_normal((1, 256, 4096)).astype(np.float32)
        w = (rng.standard_normal((256, 256, 3)) * np.sqrt(2.0 / 768)).astype(np.float32)
        fn = lambda: O.conv1d(x, w, 1, 1, nthreads=threads)
        work, unit, sample = 2.0 * 256 * 256 * 3 * 4096 / 1e12, "TFLOP/s", "1 of the 64 batch entries"
    elif wl == "pool":
        x = rng.standard_normal((2, 256, 112, 112)).astype(np.float32)
        parts = np.array_split(x.reshape(-1, 112, 112), max(1, threads))
        fn = lambda: _split_run(lambda p: O.pool2d(p, (3, 3), (2, 2), (1, 1), is_max=True), parts, threads)
        work, unit, sample = 4.0 * (x.size + x.size // 4) / 1e9, "GB/s", "2 of the 64 batch entries"
    elif wl == "batchnorm":
        x = rng.standard_normal((8, 256, 56 * 56)).astype(np.float32)
        gm = np.ones(256, np.float32)
        bt = np.zeros(256, np.float32)
        fn = lambda: O.batchnorm(x, 8, 256, 56 * 56, 1e-5, gm, bt)
        work, unit, sample = 8.0 * x.size / 1e9, "GB/s", "8 of the 64 batch entries (1 thread: per-channel loop)"
    elif wl == "mlp":
        from oracle import mlp as OM
        Ws, bs = OM.xavier_params([784, 256, 128, 10])
        data = OM.batches(4, 128, 784, 10)
        fn = lambda: OM.train([w.copy() for w in Ws], [b.copy() for b in bs], data, nthreads=threads)
        work, unit, sample = 4 * 128, "samples/s", "4 training steps of batch 128"
    elif wl == "wide_mlp":
        rows = 1
        widths = [8192] * 5 + [1000]
        Ws = [rng.uniform(-0.01, 0.01, (widths[i], widths[i + 1])).astype(np.float32) for i in range(5)]
        xs = [rng.standard_normal((rows, widths[i])).astype(np.float32) for i in range(5)]
        ds = [rng.standard_normal((rows, widths[i + 1])).astype(np.float32) for i in range(5)]

        def fn():
            for i in range(5):
                O.matmul(xs[i], Ws[i], nthreads=threads)                  # forward
                O.matmul(ds[i], np.ascontiguousarray(Ws[i].T), nthreads=threads)  # dX
                O.matmul(np.ascontiguousarray(xs[i].T), ds[i], nthreads=threads)  # dW
        work, unit, sample = rows, "samples/s", f"{rows} sample through the 15 GEMMs of one step (elementwise parts left out)"
    else:
        return None
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s or reps >= 1000:
            break
    per = dt / reps
    return work / per, unit, per, f"{sample}, {reps} repetition(s) of {per:.3f} s on {par}"


def attach_cpu_baseline(line, args, threads=1):
    r = cpu_measure(args, threads)
    if r is None:
        return
    value, unit, _, sample = r
    line["cpu_baseline"] = {"value": round(value, 6), "unit": unit, "cores": threads, "kind": "port",
                            "sample": sample + " (oracle restatement of the reference CPU loop; the reference is "
                                               "single-threaded)"}


def measure_e2e(jx, torch, dist, st, inputs, outputs, step, steps):
    """End to end through the C ABI: per step, jx_memcpy_h2d of every input
    from pinned host memory, the step, jx_memcpy_d2h of every output into
    pinned host memory; CUDA events on the launching stream, max over ranks.
    Returns (ms per step, h2d bytes per step, d2h bytes per step)."""
    s = st.cuda_stream
    hin = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in inputs]
    for h, d in zip(hin, inputs):
        h.copy_(d.cpu())
    hout = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outputs]
    nin = [t.numel() * t.element_size() for t in inputs]
    nout = [t.numel() * t.element_size() for t in outputs]

    def one():
        for h, d, nb in zip(hin, inputs, nin):
            jx.call("jx_memcpy_h2d", d.data_ptr(), h.data_ptr(), nb, s)
        step()
        for h, d, nb in zip(hout, outputs, nout):
            jx.call("jx_memcpy_d2h", h.data_ptr(), d.data_ptr(), nb, s)

    one()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        one()
    e1.record(st)
    torch.cuda.synchronize()
    return dist.max(e0.elapsed_time(e1) / steps), sum(nin), sum(nout)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_sgemm(args, dist, jx, torch):
    N = K = args.size
    M = shard(args.size, dist, "sgemm rows") if args.strong else args.size
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(1 + dist.rank)
    A = torch.empty((M, K), device=dev).uniform_(-1, 1, generator=g)   # this rank's row shard
    g.manual_seed(1)
    B = torch.empty((K, N), device=dev).uniform_(-1, 1, generator=g)   # replicated
    Cm = torch.empty((M, N), device=dev)
    gprec = jx.PREC_3XTF32_PAIR if args.gemm_prec == "pair" else jx.PREC_3XTF32
    # one launch of the SM-pair kernel per step where it applies, else the
    # split passes and the main kernel on pre-split operands
    pair = args.gemm_prec == "pair" or pair_ok(M, N, K, False, False)

    def step():
        jx.gemm(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), M, N, K, precision=gprec, stream=s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    clocks = clk.stop()
    dist.barrier()
    torch.cuda.synchronize()
    ms_max = dist.max(ms)
    flops_rank = 2.0 * M * N * K
    value = flops_rank * dist.world / (ms_max * 1e-3) / 1e12

    if pair:
        # the step is one launch of the dominant kernel: its time is the step's
        kern_ms, kern_name = ms, "gemm_pair_kernel (tcgen05 cta_group::2, split in shared memory)"
    else:
        # dominant kernel alone: the tcgen05 main loop on pre-split operands
        Kp = jx.gemm_kpad(K)
        Ah, Al = torch.empty((M, Kp), device=dev), torch.empty((M, Kp), device=dev)
        Bh, Bl = torch.empty((N, Kp), device=dev), torch.empty((N, Kp), device=dev)
        jx.gemm_split(A.data_ptr(), Ah.data_ptr(), Al.data_ptr(), M, K, stream=s)
        jx.gemm_split(B.data_ptr(), Bh.data_ptr(), Bl.data_ptr(), N, K, ld=N, trans=True, stream=s)
        for _ in range(3):
            jx.gemm_presplit(Ah.data_ptr(), Al.data_ptr(), Bh.data_ptr(), Bl.data_ptr(), Cm.data_ptr(), M, N, Kp,
                             stream=s)
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(args.steps):
            jx.gemm_presplit(Ah.data_ptr(), Al.data_ptr(), Bh.data_ptr(), Bl.data_ptr(), Cm.data_ptr(), M, N, Kp,
                             stream=s)
        e1.record(st)
        torch.cuda.synchronize()
        kern_ms, kern_name = e0.elapsed_time(e1) / args.steps, "gemm_3xtf32_kernel"
        del Ah, Al, Bh, Bl

    # e2e: host buffers through the C ABI (jx_gemm_f32_host): per step, B and
    # the row blocks of A go up from pinned host memory and C comes back,
    # overlapped with the products on three streams
    hA = torch.empty((M, K), dtype=torch.float32).pin_memory()
    hB = torch.empty((K, N), dtype=torch.float32).pin_memory()
    hC = torch.empty((M, N), dtype=torch.float32).pin_memory()
    hA.copy_(A.cpu())
    hB.copy_(B.cpu())
    nbA, nbB, nbC = hA.numel() * 4, hB.numel() * 4, hC.numel() * 4

    def e2e_step():
        jx.call("jx_gemm_f32_host", hA.data_ptr(), hB.data_ptr(), hC.data_ptr(), M, N, K, K, N, N, 0, s)

    e2e_step()
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = dist.max(e0.elapsed_time(e1) / args.e2e_steps)
    e2e_val = flops_rank * dist.world / (e2e_ms * 1e-3) / 1e12

    hbm, bf16, basis = load_peaks(clocks, ms_max * args.steps)
    peak = bf16 / 2.0 / 3.0  # tf32 issues at half the bf16 rate; 3xTF32 needs 3 MMAs per f32 product
    achieved = flops_rank / (kern_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
        "higher_is_better": True, "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic U(-1,1) operands (torch generator, seed 1)",
        "config": {"workload": f"sgemm {M}x{N}x{K} f32 per rank (M-row shard of a {M * dist.world}x{N}x{K} "
                               f"product, B replicated), JX_PREC_3XTF32",
                   "global_batch": None, "seq_len": None, "parallelism": f"M-row shards x{dist.world}, no collective",
                   "l2": f"operands {M * K * 4 / 2**20:.0f} and {K * N * 4 / 2**20:.0f} MiB; "
                         + ("> 126 MB L2, no flush needed" if M * K * 4 > 126e6 else "B re-read from L2 across steps")},
        "roofline": {"bound": "tensor", "kernel": kern_name, "achieved": round(achieved, 2),
                     "peak": round(peak, 2), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_basis": f"{basis} bf16 {bf16} TFLOP/s / 2 (tf32 rate) / 3 (3 MMAs per product)",
                     "frac_at_run_clock": at_run_clock(achieved, clocks),
                     "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS, "kernel_ms": round(kern_ms, 4)},
        "e2e": {"value": round(e2e_val, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": nbA + nbB,
                "d2h_bytes_per_step": nbC, "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": (1 if pair else 3) * args.steps,
        "clocks": clocks,
    }
    return line


def run_chain(args, dist, jx, torch):
    """chain: the fused forward y = gelu(x*a+b)*sigmoid(x) - tanh(x)/2 as a
    hand-written op-tape.  chain_grad: value_and_grad of the same function
    through the tracer (forward + VJP with a ones cotangent), y and dx out."""
    n = 1 << 28
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(2 + dist.rank)
    X = torch.randn(n, device=dev, generator=g)
    Y = torch.empty_like(X)
    grad = args.workload == "chain_grad"
    if grad:
        tr = importlib.import_module("jax-rs_b200.trace")
        DX = torch.empty_like(X)
        prog = tr.value_and_grad(lambda x: tr.gelu(x * 1.1 + 0.9) * tr.sigmoid(x) - tr.tanh(x) / 2, 1)

        def step():
            prog.run([X.data_ptr()], [Y.data_ptr(), DX.data_ptr()], n, s)
    else:
        U, B = jx.OP_UNARY, jx.OP_BINARY
        code = [(jx.OP_CONST, 1, 0, 0), (jx.OP_CONST, 2, 1, 0), (jx.OP_CONST, 3, 2, 0),
                (B + jx.BIN["mul"], 4, 0, 1), (B + jx.BIN["add"], 4, 4, 2), (U + jx.UN["gelu"], 4, 4, 0),
                (U + jx.UN["sigmoid"], 5, 0, 0), (B + jx.BIN["mul"], 4, 4, 5), (U + jx.UN["tanh"], 5, 0, 0),
                (B + jx.BIN["div"], 5, 5, 3), (B + jx.BIN["sub"], 4, 4, 5), (jx.OP_STORE, 0, 4, 0)]
        tape = jx.Tape(code, [1.1, 0.9, 2.0], 1, 1)

        def step():
            tape.run([X.data_ptr()], [Y.data_ptr()], n, s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / args.steps)
    clocks = clk.stop()
    bytes_step = (12.0 if grad else 8.0) * n
    gbs = bytes_step * dist.world / (ms * 1e-3) / 1e9
    hbm, _, basis = load_peaks()
    if grad:
        e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, [X], [Y, DX], step, args.e2e_steps)
    else:
        # e2e through jx_tape_run_host: 32 MiB blocks of x up, y down, overlapped
        hX = torch.empty_like(X, device="cpu").pin_memory()
        hX.copy_(X.cpu())
        hY = torch.empty_like(hX).pin_memory()
        ia = (jx.C.c_void_p * 1)(hX.data_ptr())
        oa = (jx.C.c_void_p * 1)(hY.data_ptr())

        def host_step():
            jx.call("jx_tape_run_host", tape.handle, ia, oa, n, 0, s)
        e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, [], [], host_step, args.e2e_steps)
        e_in, e_out = hX.numel() * 4, hY.numel() * 4
    return {"metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)",
            "config": {"workload": ("value_and_grad (tracer) of y=gelu(x*a+b)*sigmoid(x)-tanh(x)/2, y and dx, "
                                    "over 2^28 f32 per rank" if grad else
                                    "jit tape y=gelu(x*a+b)*sigmoid(x)-tanh(x)/2 over 2^28 f32 per rank"),
                       "l2": "1 GiB in + 1 GiB out > L2", "bytes_per_element": 12 if grad else 8},
            "roofline": {"bound": "hbm", "kernel": "jx_tape_kernel", "achieved": round(gbs / dist.world, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(gbs / dist.world / hbm, 4),
                         "peak_basis": basis, "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS},
            "e2e": {"value": round(bytes_step * dist.world / (e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": e_in, "d2h_bytes_per_step": e_out, "ms_per_step": round(e_ms, 3)},
            "gpu_launches": args.steps, "clocks": clocks}


def run_rng(args, dist, jx, torch):
    """uniform_range(key, [2^28], -1, 1) on the device: the reference's host
    stream reproduced by jump-ahead (4 B written per value)."""
    n = 1 << 28
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    Y = torch.empty(n, device=dev)
    key = jx.key_split(jx.key_from_seed(1 + dist.rank))[0]

    def step():
        jx.call("jx_random_uniform_f32", key[0], key[1], Y.data_ptr(), n, -1.0, 1.0, s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / args.steps)
    clocks = clk.stop()
    bytes_step = 4.0 * n
    gbs = bytes_step * dist.world / (ms * 1e-3) / 1e9
    hbm, _, basis = load_peaks()
    e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, [], [Y], step, args.e2e_steps)
    return {"metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 state -> f32", "data": "PRNGKey::from_seed(1).split().0 stream",
            "config": {"workload": "uniform_range(key, [2^28], -1, 1) per rank (xorshift128+ stream, jump-ahead)",
                       "l2": "1 GiB out > L2"},
            "roofline": {"bound": "hbm", "kernel": "rng_kernel", "achieved": round(gbs / dist.world, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(gbs / dist.world / hbm, 4),
                         "peak_basis": basis, "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS},
            "e2e": {"value": round(bytes_step * dist.world / (e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": e_in, "d2h_bytes_per_step": e_out, "ms_per_step": round(e_ms, 3)},
            "gpu_launches": args.steps, "clocks": clocks}


def run_reduce(args, dist, jx, torch):
    """Last-axis sum / argmax over [65536, 4096], or the full sum of 2^28."""
    rows, cols = 65536, 4096
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(2 + dist.rank)
    X = torch.randn((rows, cols), device=dev, generator=g)
    out = torch.empty(rows, device=dev)
    idx = torch.empty(rows, dtype=torch.int32, device=dev)
    if args.workload == "rowsum":
        def step():
            jx.reduce_axis(X.data_ptr(), out.data_ptr(), rows, cols, 1, "sum", s)
        kern, bytes_step = "reduce_rows_kernel", 4.0 * rows * cols + 4.0 * rows
    elif args.workload == "argmax":
        def step():
            jx.argreduce_rows(X.data_ptr(), idx.data_ptr(), None, rows, cols, True, s)
        kern, bytes_step = "argreduce_rows_kernel", 4.0 * rows * cols + 4.0 * rows
    elif args.workload == "sum_vjp":
        # cotangent of sum over axis 1 broadcast back: read ct [rows], write dx [rows, cols]
        CT = torch.randn(rows, device=dev, generator=g)
        DX = torch.empty_like(X)

        def step():
            jx.sum_rows_vjp(CT.data_ptr(), DX.data_ptr(), rows, cols, s)
        kern, bytes_step = "sum_rows_vjp", 4.0 * rows + 4.0 * rows * cols
    elif args.workload == "max_vjp":
        # max over axis 1: the cotangent split over the tied maxima of each row
        CT = torch.randn(rows, device=dev, generator=g)
        DX = torch.empty_like(X)

        def step():
            jx.max_rows_vjp(X.data_ptr(), CT.data_ptr(), DX.data_ptr(), rows, cols, s)
        kern, bytes_step = "max_rows_vjp", 4.0 * rows * cols + 4.0 * rows + 4.0 * rows * cols
    else:
        def step():
            jx.reduce_all(X.data_ptr(), out.data_ptr(), rows * cols, "sum", s)
        kern, bytes_step = "reduce_all_pass1", 4.0 * rows * cols
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / args.steps)
    clocks = clk.stop()
    gbs = bytes_step * dist.world / (ms * 1e-3) / 1e9
    hbm, _, basis = load_peaks()
    if args.workload in ("sum_vjp", "max_vjp"):
        ins = [CT] if args.workload == "sum_vjp" else [X, CT]
        e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, ins, [DX], step, args.e2e_steps)
    else:
        res = [idx] if args.workload == "argmax" else ([out] if args.workload == "rowsum" else [out[:1]])
        e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, [X], res, step, args.e2e_steps)
    return {"metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)",
            "config": {"workload": f"{args.workload} over [{rows}, {cols}] f32 per rank",
                       "l2": "1 GiB input or output > L2"},
            "e2e": {"value": round(bytes_step * dist.world / (e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": e_in, "d2h_bytes_per_step": e_out, "ms_per_step": round(e_ms, 3)},
            "roofline": {"bound": "hbm", "kernel": kern, "achieved": round(gbs / dist.world, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(gbs / dist.world / hbm, 4), "peak_basis": basis,
                         "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS},
            "gpu_launches": args.steps * (2 if args.workload == "fullsum" else 1), "clocks": clocks}


def run_conv_bgemm(args, dist, jx, torch):
    """conv: [64,256,56,56] x [256,256,3,3] stride 1 pad 1, forward + dX + dW per step.
    bgemm: batched [64,2048,2048] x [64,2048,2048] (einsum bij,bjk->bik)."""
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(3 + dist.rank)
    if args.workload == "conv":
        jx.call("jx_conv_set_kernel", {"auto": jx.CONV_AUTO, "one_cta": jx.CONV_ONE_CTA, "pair": jx.CONV_PAIR}[args.conv_kernel])
        Bg = args.conv_batch or 64  # global batch, split over the ranks
        B, C, H, W, O, K = shard(Bg, dist, "conv batch"), 256, 56, 56, 256, 3
        geo = (B, C, H, W, O, K, K, 1, 1)
        X = torch.randn((B, C, H, W), device=dev, generator=g)
        Wt = torch.randn((O, C, K, K), device=dev, generator=g) * float(np.sqrt(2.0 / (C * K * K)))
        G = torch.randn((B, O, H, W), device=dev, generator=g)
        Y, DX, DW = torch.empty_like(G), torch.empty_like(X), torch.empty_like(Wt)

        def step():
            jx.call("jx_conv2d_fwd_f32", X.data_ptr(), Wt.data_ptr(), Y.data_ptr(), *geo, s)
            jx.call("jx_conv2d_bwd_data_f32", G.data_ptr(), Wt.data_ptr(), DX.data_ptr(), *geo, s)
            jx.call("jx_conv2d_bwd_filter_f32", X.data_ptr(), G.data_ptr(), DW.data_ptr(), *geo, s)
        flops = 3 * 2.0 * B * O * C * K * K * H * W
        wl = (f"conv2d [{Bg},256,56,56] x [256,256,3,3] s1 p1: forward + input grad + weight grad per step, "
              f"{B} images per rank (per-rank weight-gradient partials, no collective)")
    else:
        nb, n = shard(64, dist, "bgemm batch"), 2048
        A = torch.empty((nb, n, n), device=dev).uniform_(-1, 1, generator=g)
        Bm = torch.empty((nb, n, n), device=dev).uniform_(-1, 1, generator=g)
        Cm = torch.empty((nb, n, n), device=dev)

        gprec = jx.PREC_3XTF32_PAIR if args.gemm_prec == "pair" else jx.PREC_3XTF32

        def step():
            jx.gemm(A.data_ptr(), Bm.data_ptr(), Cm.data_ptr(), n, n, n, batch=nb, strideA=n * n, strideB=n * n,
                    strideC=n * n, precision=gprec, stream=s)
        flops = 2.0 * nb * n ** 3
        wl = (f"batched sgemm [64,2048,2048] x [64,2048,2048] (einsum bij,bjk->bik), {nb} batch entries per rank, "
              "JX_PREC_3XTF32")
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / args.steps)
    clocks = clk.stop()
    tf = flops * dist.world / (ms * 1e-3) / 1e12
    _, bf16, basis = load_peaks(clocks, ms * args.steps)
    peak = bf16 / 2.0 / 3.0
    if args.workload == "conv":
        e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, [X, Wt, G], [Y, DX, DW], step, args.e2e_steps)
    else:
        # through the host-buffer entry point: batch blocks stream up, multiply and down overlapped
        hA, hB = A.cpu().pin_memory(), Bm.cpu().pin_memory()
        hC = torch.empty(Cm.shape).pin_memory()

        def host_step():
            jx.call("jx_gemm_batched_f32_host", hA.data_ptr(), hB.data_ptr(), hC.data_ptr(), n, n, n, nb, 0, s)
        e_ms = time_host_steps(torch, dist, st, host_step, args.e2e_steps)
        e_in, e_out = 2 * hA.numel() * 4, hC.numel() * 4
    return {"metric": METRIC, "value": round(tf, 2), "unit": "TFLOP/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl, "parallelism": f"global batch split over {dist.world} rank(s), no collective"},
            "roofline": {"bound": "tensor",
                         "kernel": (("conv_gemm_kernel x3 (implicit GEMM, one CTA" if args.conv_kernel == "one_cta"
                                     else "conv_pair_kernel x3 (implicit GEMM on SM pairs")
                                    + "; whole step incl. filter/dY splits)"
                                    if args.workload == "conv" else
                                    ("gemm_pair_kernel" if pair_ok(2048, 2048, 2048, False, False, nb)
                                     else "gemm_fused_split_kernel") + " (whole batched call)"),
                         "achieved": round(tf / dist.world, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                         "frac": round(tf / dist.world / peak, 4), "peak_basis": f"{basis} bf16 / 2 / 3",
                         "frac_at_run_clock": at_run_clock(tf / dist.world, clocks),
                         "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS},
            "e2e": {"value": round(flops * dist.world / (e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": e_in, "d2h_bytes_per_step": e_out, "ms_per_step": round(e_ms, 3)},
            "gpu_launches": args.steps * (10 if args.workload == "conv" else
                                          gemm_kernels(2048, 2048, 2048, False, False, False, batch=nb)),
            "clocks": clocks}


def run_layers(args, dist, jx, torch):
    """conv1d: [64,256,4096] x [256,256,3] stride 1 pad 1 (exact f32, the
    reference's summation order).  pool: 3x3 stride-2 pad-1 max pooling of
    [64,256,112,112].  batchnorm: batch_norm_2d of [64,256,56,56] with gamma
    and beta (statistics, then normalisation)."""
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(5 + dist.rank)
    B = args.conv_batch or 64
    if args.workload == "conv1d":
        C = O = 256
        L, K = 4096, 3
        X = torch.randn((B, C, L), device=dev, generator=g)
        Wt = torch.randn((O, C, K), device=dev, generator=g) * float(np.sqrt(2.0 / (C * K)))
        Y = torch.empty((B, O, L), device=dev)

        def step():
            jx.call("jx_conv1d_f32", X.data_ptr(), Wt.data_ptr(), Y.data_ptr(), B, C, O, L, K, 1, 1, s)
        work = 2.0 * B * O * C * K * L
        ins, outs, launches = [X, Wt], [Y], 1
        wl = f"conv1d [{B},256,4096] x [256,256,3] stride 1 pad 1, exact f32 (unfused multiply-add)"
    elif args.workload == "pool":
        C, H = 256, 112
        X = torch.randn((B, C, H, H), device=dev, generator=g)
        OH = (H + 2 - 3) // 2 + 1
        Y = torch.empty((B, C, OH, OH), device=dev)

        def step():
            jx.call("jx_maxpool2d_f32", X.data_ptr(), Y.data_ptr(), B, C, H, H, 3, 3, 2, 1, s)
        work = 4.0 * (X.numel() + Y.numel())
        ins, outs, launches = [X], [Y], 1
        wl = f"maxpool2d 3x3 stride 2 pad 1 over [{B},256,112,112] -> [{B},256,56,56]"
    else:
        C, HW = 256, 56 * 56
        X = torch.randn((B, C, HW), device=dev, generator=g) * 2.0 + 0.5
        Gm = torch.empty(C, device=dev).uniform_(0.5, 1.5, generator=g)
        Bt = torch.randn(C, device=dev, generator=g)
        Y = torch.empty_like(X)

        def step():
            jx.call("jx_batchnorm_f32", X.data_ptr(), Gm.data_ptr(), Bt.data_ptr(), Y.data_ptr(), B, C, HW, 1e-5,
                    None, None, s)
        work = 8.0 * X.numel()
        ins, outs, launches = [X, Gm, Bt], [Y], 3
        wl = f"batch_norm_2d [{B},256,56,56] with gamma, beta (statistics + normalisation)"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / args.steps)
    clocks = clk.stop()
    if args.workload == "pool":
        hX = X.cpu().pin_memory()
        hY = torch.empty(Y.shape).pin_memory()

        def host_step():
            jx.call("jx_pool2d_f32_host", hX.data_ptr(), hY.data_ptr(), B, C, H, H, 3, 3, 2, 2, 1, 1,
                    jx.POOL_MAX, 0, s)
        e_ms = time_host_steps(torch, dist, st, host_step, args.e2e_steps)
        e_in, e_out = hX.numel() * 4, hY.numel() * 4
    else:
        e_ms, e_in, e_out = measure_e2e(jx, torch, dist, st, ins, outs, step, args.e2e_steps)
    hbm, _, basis = load_peaks()
    if args.workload == "conv1d":
        val = work * dist.world / (ms * 1e-3) / 1e12
        e2e = work * dist.world / (e_ms * 1e-3) / 1e12
        unit = "TFLOP/s"
        mhz = clocks.get("sm_max_mhz") or 1965.0
        peak = 148 * 128 * mhz * 1e6 / 1e12
        roof = {"bound": "fp32 issue", "kernel": "conv1d_kernel", "achieved": round(val / dist.world, 2),
                "peak": round(peak, 2), "unit": "TFLOP/s", "frac": round(val / dist.world / peak, 4),
                "peak_basis": f"nominal: 148 SMs x 128 FP32 lanes x {mhz:.0f} MHz, one flop per unfused FMUL or "
                              "FADD (no measured FP32 peak)", "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS}
    else:
        val = work * dist.world / (ms * 1e-3) / 1e9
        e2e = work * dist.world / (e_ms * 1e-3) / 1e9
        unit = "GB/s"
        roof = {"bound": "hbm", "kernel": "pool2d_kernel" if args.workload == "pool" else
                "norm_stats_wide + norm_finalize + norm_apply (whole call)",
                "achieved": round(val / dist.world, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(val / dist.world / hbm, 4), "peak_basis": basis, "traffic": traffic_for(args, dist.world),
                "traffic_basis": TRAFFIC_BASIS,
                "note": "algorithmic bytes: one read of x and one write of y" +
                        ("; the statistics need a second read of x (12 B per element moved at best without L2 "
                         "reuse), so 8 B per element is a floor no two-pass kernel reaches"
                         if args.workload == "batchnorm" else "")}
    return {"metric": METRIC, "value": round(val, 2), "unit": unit, "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) (torch generator)",
            "config": {"workload": wl, "l2": "input > L2", "parallelism": f"batch shards x{dist.world}"},
            "roofline": roof,
            "e2e": {"value": round(e2e, 2), "unit": unit, "h2d_bytes_per_step": e_in, "d2h_bytes_per_step": e_out,
                    "ms_per_step": round(e_ms, 3)},
            "gpu_launches": args.steps * launches, "clocks": clocks}


def time_host_steps(torch, dist, st, host_step, steps):
    """ms per call of a host-buffer entry point (copies inside), CUDA events on
    the caller's stream (which waits for the call's last download), max over
    ranks."""
    host_step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        host_step()
    e1.record(st)
    torch.cuda.synchronize()
    return dist.max(e0.elapsed_time(e1) / steps)


def run_fft(args, dist, jx, torch):
    """Batched complex FFTs: 1-D n=4096 x 65536, or 2-D 1024x1024 x 256 per rank."""
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(3 + dist.rank)
    if args.workload == "fft1d":
        n, batch = 4096, shard(args.fft_batch or 65536, dist, "FFT batch")
        X = torch.randn((batch, n, 2), device=dev, generator=g)
        Y = torch.empty_like(X)

        def step():
            jx.fft_c2c(X.data_ptr(), Y.data_ptr(), n, batch, False, s)
        wl, kern, launches = (f"1-D complex FFT n={n} x batch {batch * dist.world}, {batch} transforms per rank",
                              "fft_kernel", 1)
    else:
        h = w = 1024
        batch = shard(args.fft_batch or 256, dist, "FFT batch")
        X = torch.randn((batch, h, w, 2), device=dev, generator=g)
        Y = torch.empty_like(X)

        def step():
            jx.fft2_c2c(X.data_ptr(), Y.data_ptr(), h, w, batch, False, s)
        wl, kern, launches = (f"2-D complex FFT {h}x{w} x batch {batch * dist.world}, {batch} images per rank "
                              "(rows, then columns)", "fft_kernel", 2)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / args.steps)
    clocks = clk.stop()
    nbytes = 2.0 * X.numel() * 4  # algorithmic: one read and one write of the batch
    gbs = nbytes * dist.world / (ms * 1e-3) / 1e9
    kern_ms, kern_note = ms, ""
    if launches == 2:
        # The column pass alone: the row pass is the same kernel launch as a
        # batched 1-D transform of the h*batch rows, timed the same way.
        for _ in range(args.warmup):
            jx.fft_c2c(X.data_ptr(), Y.data_ptr(), w, h * batch, False, s)
        e0.record(st)
        for _ in range(args.steps):
            jx.fft_c2c(X.data_ptr(), Y.data_ptr(), w, h * batch, False, s)
        e1.record(st)
        torch.cuda.synchronize()
        row_ms = e0.elapsed_time(e1) / args.steps
        kern_ms = max(ms - row_ms, 1e-6)
        kern, kern_note = "fft1024_tma_kernel (column pass)", f"row pass {row_ms:.4f} ms, column pass {kern_ms:.4f} ms"
    hbm, _, basis = load_peaks()
    kgbs = nbytes / (kern_ms * 1e-3) / 1e9
    # e2e through the host-buffer FFT entry points: blocks of transforms go up,
    # come back, overlapped with the transforms on three streams
    hX = torch.empty_like(X, device="cpu").pin_memory()
    hX.copy_(X.cpu())
    hY = torch.empty_like(hX).pin_memory()
    if launches == 2:
        host_step = lambda: jx.call("jx_fft2_c2c_f32_host", hX.data_ptr(), hY.data_ptr(), h, w, batch, 0, 0, s)
    else:
        host_step = lambda: jx.call("jx_fft_c2c_f32_host", hX.data_ptr(), hY.data_ptr(), n, batch, 0, 0, s)
    e_ms, _, _ = measure_e2e(jx, torch, dist, st, [], [], host_step, args.e2e_steps)
    e_in, e_out = hX.numel() * 4, hY.numel() * 4
    return {"metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (complex64)", "data": "synthetic N(0,1) real and imaginary parts",
            "config": {"workload": wl, "l2": f"{nbytes / 2 / 2**30:.2f} GiB per pass per rank",
                       "parallelism": f"global batch split over {dist.world} rank(s), no collective"},
            "roofline": {"bound": "hbm", "kernel": kern, "achieved": round(kgbs, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(kgbs / hbm, 4), "peak_basis": basis,
                         "traffic": traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS, "kernel_ms": round(kern_ms, 4), "note": kern_note},
            "e2e": {"value": round(nbytes * dist.world / (e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": e_in, "d2h_bytes_per_step": e_out, "ms_per_step": round(e_ms, 3)},
            "gpu_launches": args.steps * launches, "clocks": clocks}


def pair_ok(M, N, K, transA, transB, batch=1, sms=148):
    """Whether jx_gemm_f32 (JX_PREC_3XTF32) takes the SM-pair kernel: leading
    dimensions (contiguous operands) multiples of 4 floats and at least one
    256x256 tile per SM pair."""
    lda = M if transA else K
    ldb = K if transB else N
    return lda % 4 == 0 and ldb % 4 == 0 and -(-M // 256) * -(-N // 256) * batch >= sms // 2


def gemm_kernels(M, N, K, transA, transB, exact, batch=1, sms=148):
    """Kernels one jx_gemm_f32 call launches: 1 (exact, the SM-pair kernel, or
    the fused-split kernel: untransposed rows of multiples of 4 floats,
    250*(1/M + 1/N) > 0.2, at least one 128x256 tile per SM) or 3 (two tf32
    split passes + the tcgen05 kernel)."""
    if exact or pair_ok(M, N, K, transA, transB, batch, sms):
        return 1
    tiles = -(-M // 128) * -(-N // 256) * batch
    fused = (not transA and not transB and K % 4 == 0 and N % 4 == 0 and 250.0 * (1.0 / M + 1.0 / N) > 0.2
             and tiles >= sms)
    return 1 if fused else 3


def mlp_launches(widths, batch, exact, dp=False):
    """Kernels in one jx_mlp_train_step: forward GEMM + bias/activation per
    layer; softmax-xent (2); backward dW GEMM (A transposed) + column sums (2)
    per layer, dh GEMM (B transposed) + activation backward below the top
    layer; Adam + step counter (2).  Data parallel (dp): one Adam launch per
    layer bucket, and layer 1's weight gradient as column sums (2) + one GEMM
    per row chunk (2) when its width splits into two multiples of 128 (NCCL's
    own kernels are not counted)."""
    L, n = len(widths) - 1, 4
    for l in range(L):
        K, N = widths[l], widths[l + 1]
        n += gemm_kernels(batch, N, K, False, False, exact) + 1
        if dp and l == 0 and not exact and K % 256 == 0:
            n += 2 + 2 * gemm_kernels(K // 2, N, batch, True, False, exact)
        else:
            n += gemm_kernels(K, N, batch, True, False, exact) + 2
        if l > 0:
            n += gemm_kernels(batch, K, N, False, True, exact) + 1
    if dp:
        n += L - 1
    return n


def run_mlp(args, dist, jx, torch, steps=None, warmup=None, e2e=True):
    """MLP training through the native trainer (jx_mlp_train_step).

    mlp:      784-256-128-10 ReLU, batch 128, Adam; one GPU (replicas for N > 1).
    wide_mlp: 8192 -> 4 x (8192 GELU) -> 1000, global batch split over the
              ranks, gradients all-reduced per layer with NCCL (data parallel).
    """
    wide = args.workload == "wide_mlp" or steps is not None
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    if wide:
        widths, acts = [8192, 8192, 8192, 8192, 8192, 1000], ["gelu"] * 4
        gb = args.global_batch
        assert gb % dist.world == 0, "global batch must divide by the rank count"
        batch = gb // dist.world
    else:
        widths, acts, batch = [784, 256, 128, 10], ["relu", "relu"], 128
        gb = batch * dist.world
    if args.precision is None:
        args.precision = "3xtf32" if wide else "exact"
    prec = jx.PREC_EXACT if args.precision == "exact" else jx.PREC_3XTF32
    dev = torch.device("cuda", dist.local)
    st = torch.cuda.current_stream()
    s = st.cuda_stream
    net = jx.MLP(widths, acts, batch, prec)
    rng = np.random.default_rng(1)  # identical initial parameters on every rank
    Ws, bs = [], []
    for l in range(len(widths) - 1):
        fi, fo = widths[l], widths[l + 1]
        if wide:  # He-normal
            Ws.append((rng.standard_normal((fi, fo), dtype=np.float32) * np.float32(np.sqrt(2.0 / fi))))
        else:  # Xavier-uniform
            a = np.sqrt(6.0 / (fi + fo))
            Ws.append(rng.uniform(-a, a, (fi, fo)).astype(np.float32))
        bs.append(np.zeros(fo, np.float32))
    net.set_params(net.pack(Ws, bs))
    net.set_adam(1e-3, 0.9, 0.999, 1e-8)
    comm = None
    if dist.world > 1 and wide:
        import ctypes as C
        nid = jx.lib().jx_nccl_unique_id_size()
        idb = (C.c_char * nid)()
        if dist.rank == 0:
            jx.call("jx_nccl_get_unique_id", idb)
        obj = [bytes(idb)]
        dist.pg.broadcast_object_list(obj, src=0)
        idb = (C.c_char * nid).from_buffer_copy(obj[0])
        comm = C.c_void_p()
        jx.call("jx_nccl_init", idb, dist.world, dist.rank, 120000, C.byref(comm))
        net.attach_comm(comm, dist.world, gb)
    # a few pre-generated batches on the device, cycled through (inputs are
    # per-step synthetic data; generating them is outside the timed region)
    g = torch.Generator(device=dev)
    g.manual_seed(100 + dist.rank)
    nb = 4
    X = [torch.randn((batch, widths[0]), device=dev, generator=g) for _ in range(nb)]
    Y = [torch.randint(0, widths[-1], (batch,), device=dev, generator=g).float() for _ in range(nb)]
    loss = torch.empty(1, device=dev)

    def step(i):
        net.step(X[i % nb].data_ptr(), Y[i % nb].data_ptr(), loss.data_ptr(), s)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(dist.local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        step(i)
    e1.record(st)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / steps)
    clocks = clk.stop()
    final_loss = float(loss.item())
    samples = gb if wide else batch * dist.world
    value = samples / (ms * 1e-3)
    # e2e: per step, the batch comes from pinned host memory and the loss goes back
    hx = torch.empty((batch, widths[0]), dtype=torch.float32).pin_memory()
    hy = torch.empty((batch,), dtype=torch.float32).pin_memory()
    hl = torch.empty((1,), dtype=torch.float32).pin_memory()
    hx.copy_(X[0].cpu())
    hy.copy_(Y[0].cpu())
    e2e_steps = max(1, min(steps, 20 if not wide else 3))
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(e2e_steps):
        jx.call("jx_memcpy_h2d", X[0].data_ptr(), hx.data_ptr(), hx.numel() * 4, s)
        jx.call("jx_memcpy_h2d", Y[0].data_ptr(), hy.data_ptr(), hy.numel() * 4, s)
        step(0)
        jx.call("jx_memcpy_d2h", hl.data_ptr(), loss.data_ptr(), 4, s)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = dist.max(e0.elapsed_time(e1) / e2e_steps)
    flops = 0.0
    for l in range(len(widths) - 1):
        # forward and weight-gradient GEMMs per layer; the input gradient
        # (dh = dz W^T) for every layer but the first
        flops += (3 if l > 0 else 2) * 2.0 * batch * widths[l] * widths[l + 1]
    _, bf16, basis = load_peaks(clocks, ms * steps)
    peak = bf16 / 2.0 / 3.0
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "samples/s", "n_gpus": dist.world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if wide else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1) inputs, uniform integer labels (torch generator)",
        "config": {"workload": ("wide MLP 8192-4x8192(GELU)-1000, softmax-CE, Adam, data parallel"
                                if wide else "MLP 784-256(ReLU)-128(ReLU)-10, softmax-CE, Adam"),
                   "global_batch": samples, "per_rank_batch": batch, "precision": args.precision,
                   "parallelism": f"dp{dist.world}" + (" (NCCL per-layer gradient all-reduce)" if wide and
                                                      dist.world > 1 else "")},
        "final_loss": final_loss,
        "roofline": {"bound": "tensor" if wide else "launch", "kernel": "whole training step",
                     "achieved": round(flops / (ms * 1e-3) / 1e12, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(flops / (ms * 1e-3) / 1e12 / peak, 4),
                     "peak_basis": f"{basis} bf16 {bf16} / 2 / 3 (3xTF32)",
                     "frac_at_run_clock": at_run_clock(flops / (ms * 1e-3) / 1e12, clocks),
                     "traffic": None if wide else traffic_for(args, dist.world), "traffic_basis": TRAFFIC_BASIS,
                     "note": ("exact f32 (sequential-k, unfused): the whole step is one cooperative kernel "
                              "with grid barriers between its phases; the tensor peak is quoted for scale")
                     if prec == jx.PREC_EXACT else ""},
        "e2e": {"value": round(samples / (e2e_ms * 1e-3), 1), "unit": "samples/s",
                "h2d_bytes_per_step": (hx.numel() + hy.numel()) * 4, "d2h_bytes_per_step": 4,
                "ms_per_step": round(e2e_ms, 4)},
        # exact precision on one GPU: the whole step is one cooperative kernel
        "gpu_launches": steps * (1 if prec == jx.PREC_EXACT and comm is None
                                      else mlp_launches(widths, batch, prec == jx.PREC_EXACT, comm is not None)),
        "clocks": clocks,
    }
    if wide:
        # where a step's time goes: CUDA events on the caller's stream around
        # the forward pass, the backward pass as enqueued there, and the tail
        # that waits for the last all-reduces and Adam updates (max over ranks)
        net.set_timing(True)
        ph = []
        for i in range(3):
            step(i)
            ph.append(net.step_times())
        net.set_timing(False)
        fw, bw, tail = (dist.max(statistics.median(p[k] for p in ph)) for k in range(3))
        line["phases_ms"] = {"forward": round(fw, 3), "backward": round(bw, 3), "tail": round(tail, 3),
                             "tail_frac": round(tail / max(fw + bw + tail, 1e-9), 4),
                             "note": "CUDA events in separate (untimed) steps; tail = exposed gradient exchange (reduce-scatter + all-gather, or all-reduce) + Adam"
                                     if comm is not None else "CUDA events in separate (untimed) steps; tail = Adam"}
    if comm is not None:
        torch.cuda.synchronize()
        del net
        jx.call("jx_nccl_destroy", comm)
    return line


def wide_mlp_sub(args, dist, jx, torch):
    """The wide-MLP data-parallel training measurement the default line
    carries beside its GEMM headline: 8192 -> 4 x 8192 (GELU) -> 1000, global
    batch 65536 split over the ranks, NCCL all-reduce of every layer's
    gradient bucket, Adam; its own warm-up (>= 3 steps) and timed steps."""
    torch.cuda.empty_cache()
    w = max(3, min(args.warmup, 5))
    k = max(3, args.wide_steps)
    sub = run_mlp(args, dist, jx, torch, steps=k, warmup=w)
    keep = ("value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "config", "final_loss",
            "roofline", "e2e", "gpu_launches", "clocks", "phases_ms")
    return {key: sub[key] for key in keep if key in sub}


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    dist = Dist(args.gpus)
    torch.cuda.set_device(dist.local)
    jx = importlib.import_module("jax-rs_b200")
    jx.init(dist.local)
    lines = []
    for wl in args.workload.split(","):
        args.workload = wl
        if wl == "sgemm":
            line = run_sgemm(args, dist, jx, torch)
            if not args.no_wide_mlp:
                try:
                    line["wide_mlp"] = wide_mlp_sub(args, dist, jx, torch)
                except Exception as e:  # keep the GEMM headline if the training run fails
                    line["wide_mlp"] = {"error": f"{type(e).__name__}: {e}"[:400]}
        elif wl in ("chain", "chain_grad"):
            line = run_chain(args, dist, jx, torch)
        elif wl == "rng":
            line = run_rng(args, dist, jx, torch)
        elif wl in ("mlp", "wide_mlp"):
            line = run_mlp(args, dist, jx, torch)
        elif wl in ("fft1d", "fft2d"):
            line = run_fft(args, dist, jx, torch)
        elif wl in ("conv", "bgemm"):
            line = run_conv_bgemm(args, dist, jx, torch)
        elif wl in ("conv1d", "pool", "batchnorm"):
            line = run_layers(args, dist, jx, torch)
        else:
            line = run_reduce(args, dist, jx, torch)
        if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
            attach_cpu_baseline(line, args, threads=1)
        lines.append(line)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    dist.close()
    if dist.rank == 0:
        for line in lines:
            print(json.dumps(line), flush=True)


def reference_arm(args):
    """The reference's CPU implementation of the same workload (the oracle's
    restatement of its loops), a bounded sample per step, on one host thread:
    the reference's CPU path is single-threaded (no rayon, no threads), so one
    thread is all it can use.  The same restatement split over every host
    thread is reported beside it as `value_all_threads`."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    args.workload = args.workload.split(",")[0]
    threads = 1
    steps = max(1, min(args.steps, 3))
    vals, pers, sample, unit = [], [], "", ""
    for _ in range(steps):
        r = cpu_measure(args, threads, budget_s=4.0)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": f"no CPU restatement for {args.workload}"}))
            return
        v, unit, per, sample = r
        vals.append(v)
        pers.append(per)
    value = statistics.median(vals)
    all_threads = os.cpu_count() or 1
    r_all = cpu_measure(args, all_threads, budget_s=4.0) if all_threads > 1 else None
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": unit, "n_gpus": args.gpus,
        "value_all_threads": {"value": round(r_all[0], 6), "cores": all_threads} if r_all else None,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(statistics.median(pers) * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload} (sample of the GPU arm's workload)"},
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads, "kind": "port",
                         "sample": sample + " (oracle restatement of the reference CPU loop; the reference is "
                                            "single-threaded)"},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
