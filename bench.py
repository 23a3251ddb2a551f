#!/usr/bin/env python
"""Benchmark of the B200 fp32 GEMM path (the reference's `gemm` + `bias_add` on CUDA).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--precision 3xtf32|1xtf32]
                    [--impl mine|reference] [--workload c2|c3|c4|c5|gemv|copy]

Workload ("C2"): per rank, C = 0.5 * A @ B^T + 1.0 * C_in + bias with
A, B, C_in [8192, 8192] ~ N(0, 1) and bias [8192] ~ U(-0.1, 0.1), fp32 in HBM, one fused call
per step (3xTF32 by default). Under torchrun every rank owns one 8192-row block of an
M = 8192*N problem with B and bias replicated, so per-GPU work is fixed ("scaling": "weak") and
there is no collective on the data path. `value` is the whole-job TFLOP/s (2*M*N*K per step
summed over ranks, divided by the max-over-ranks device time). The other workloads: `c3` (the
two-layer MLP forward, `--prepacked` for pre-split weights), `c4` (the two attention GEMMs,
batch x heads split over the ranks; `--heads` for smaller profiling cases), `c5` (32768 x 32768
x 8192, row blocks split over the ranks: strong scaling; at N > 1 the gather of C to rank 0 fused
into the GEMM is timed against NCCL's all-gather), `gemv` (65536 x 8192, HBM-bound) and `copy`
(Tensor::contiguous of an 8192^2 view on the device, `--view transpose|slice|stepped`).
Every workload reports the reference's own CPU path on a bounded sample as `cpu_baseline`.

The default C2 line also carries `sustained` (the same step back to back for ~2.5 s, with its own
clock record, against the sustained GEMM peak) and `c5` (the C5 strong-scaling GEMM at the same
N: per-N step and kernel times, and at N > 1 NCCL's all-gather of C and the gather fused into the
GEMM, with the GB/s into rank 0), so one SCALE run gives both the C2 weak and the C5 strong
scaling. The JSON line is the last line of stdout.

`--impl reference` times the reference's own CPU implementation (the unmodified library built
from its sources into oracle/_ref, public gemm + bias_add, all host threads) on the whole C2
problem every step; rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fp32 GEMM TFLOP/s (3xTF32) at 1/2/4/8 B200 and % of TF32 tensor roofline"
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--precision", choices=["3xtf32", "1xtf32"], default="3xtf32")
    p.add_argument("--impl", choices=["mine", "reference"], default="mine")
    p.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "gemv", "copy"], default="c2")
    p.add_argument("--prepacked", action="store_true",
                   help="c3: W1 and W2 split once before the timed region (pack_b), as the "
                        "reference's PackedB serves inference")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--size", type=int, default=8192,
                   help="c2 only: M = N = K per rank (profiling captures use a smaller case)")
    p.add_argument("--heads", type=int, default=512,
                   help="c4 only: batch x heads (512 in the config; profiling captures use fewer)")
    p.add_argument("--c4-unfused", action="store_true",
                   help="c4: time the two batched GEMMs of the composed path (S, then P@V with a "
                        "stand-in P) instead of the one-kernel causal attention")
    p.add_argument("--view", choices=["transpose", "slice", "stepped"], default="transpose",
                   help="copy only: the packed view (transposed; a column slice of a wider "
                        "matrix, read as 16-byte rows; every other column, a gather)")
    p.add_argument("--mnk", type=str, default=None,
                   help="c2: 'M,N,K' per rank instead of --size; gemv: 'M,1,K' (profiling shapes)")
    p.add_argument("--c5-steps", type=int, default=10,
                   help="c2 at 8192: steps of the C5 strong-scaling leg reported as `c5` beside "
                        "the C2 line (0 skips it)")
    p.add_argument("--sustained-s", type=float, default=2.5,
                   help="c2 at 8192: seconds of back-to-back steps for the `sustained` figure (0 "
                        "skips it)")
    return p.parse_args()


# What each workload's end-to-end leg times (every copy is inside the timed region).
E2E_PATHS = {
    "c2": "the public gemm on pinned host tensors (execution='gpu'): host -> device copies, the C "
          "ABI kernel, device -> host copy of C, pipelined by row blocks",
    "c5": "the public gemm on pinned host tensors (execution='gpu'): host -> device copies, the C "
          "ABI kernel, device -> host copy of C, pipelined by row blocks",
    "c3": "pinned host W1, b1, b2, X's first row block, W2 and X's other row blocks copied in "
          "(each weight split once by pack_b when it has landed), both fused linear calls on "
          "each block, its rows of Y copied back, on three streams so one block's copies "
          "overlap another's math; with --prepacked the split weights stay resident and only X "
          "and Y cross the host link",
    "c4": "the public attention op (S = QK^T/sqrt(d), causal masked softmax, O = PV) on pinned "
          "host q, k, v (execution='gpu'): batch chunks copied in, attended and O copied back, "
          "overlapped on three streams",
    "default": "pinned host inputs copied in, the op, the result copied back (one stream)",
}


# ---- peaks ------------------------------------------------------------------------------------

def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"bf16_burst": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"bf16_burst": FALLBACK_BF16_TFLOPS, "bf16_sustained": FALLBACK_BF16_TFLOPS,
                "hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback"}


def profiled_traffic(workload: str, precision: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any
    (a line `traffic_bytes_per_launch[<workload>/<precision>]: <bytes>`)."""
    pat = re.compile(r"traffic_bytes_per_launch\[(\w+)/(\w+)\]:\s*([0-9.eE+]+)")
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if not name.endswith((".md", ".txt")):
            continue
        with open(os.path.join(pdir, name)) as f:
            for line in f:
                m = pat.search(line)
                if m and m.group(1) == workload and m.group(2) == precision:
                    return float(m.group(3))
    return None


# ---- clocks -----------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi sampled every 100 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
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
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)], stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) == 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---- distributed plumbing -------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def emit(obj):
    print(json.dumps(obj), flush=True)


# ---- the reference arm / CPU baseline ----------------------------------------------------------

def host_threads() -> int:
    """Every host CPU this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_gemm_sample(m_full, n, k, target_s, reps, warmup=1):
    """Times the reference's own public gemm (+ bias_add) on a row sample of the C2 workload,
    with all host threads. Returns (seconds per call list, sample rows, kind, cores)."""
    from oracle import oracle as O

    ref = O.reference()
    if ref is None:
        return None
    ref.mfref_set_threads(host_threads())
    cores = int(ref.mfref_max_threads())
    rows = 64
    bench = O.RefGemmBench(rows, n, k, True, 1)
    t = float(min(bench.run(0.5, 1.0, True, 2)))
    bench.close()
    rows = int(max(64, min(m_full, (target_s / max(t, 1e-6)) * rows)) // 64 * 64)
    bench = O.RefGemmBench(rows, n, k, True, 1)
    if warmup:
        bench.run(0.5, 1.0, True, warmup)
    secs = list(bench.run(0.5, 1.0, True, reps))
    bench.close()
    return secs, rows, "reference", cores


def reference_cpu_baseline(args, m, n, k):
    """The reference's own CPU path (the unmodified library in oracle/_ref, public API, all host
    threads) on a bounded sample of the workload, in the workload's unit."""
    from oracle import oracle as O

    ref = O.reference()
    if ref is None:
        return None
    ref.mfref_set_threads(host_threads())
    cores = int(ref.mfref_max_threads())
    if args.workload == "c3":
        secs = O.ref_time_mlp(4096, 1024, 4096, 2, 1, 3)
        per = float(statistics.median(secs))
        return {"value": 2.0 * 2 * 4096 * 1024 * 4096 / per / 1e12, "unit": "TFLOP/s",
                "cores": cores, "kind": "reference",
                "sample": f"the whole C3 forward (matmul, bias_add, gelu, matmul, bias_add) on "
                          f"the reference's public API, median of 3 calls, {per * 1e3:.1f} ms each"}
    if args.workload == "c4":
        heads = 8
        secs = O.ref_time_attention_gemms(heads, 2048, 128, 3, 1, 3)
        per = float(statistics.median(secs))
        return {"value": 2.0 * 2 * heads * 2048 * 2048 * 128 / per / 1e12, "unit": "TFLOP/s",
                "cores": cores, "kind": "reference",
                "sample": f"{heads} of 512 heads: the two gemm_strided_batched calls, median of 3, "
                          f"{per * 1e3:.1f} ms each"}
    if args.workload == "c5":
        rows = 512
        bench = O.RefGemmBench(rows, 32768, 8192, False, 4)
        bench.run(1.0, 0.0, False, 1)
        secs = list(bench.run(1.0, 0.0, False, 3))
        bench.close()
        per = float(statistics.median(secs))
        return {"value": 2.0 * rows * 32768 * 8192 / per / 1e12, "unit": "TFLOP/s",
                "cores": cores, "kind": "reference",
                "sample": f"{rows} of 32768 rows of A/C (B full), median of 3 gemm calls, "
                          f"{per:.2f} s each"}
    rows = 16384
    secs = O.ref_time_gemv(rows, 8192, 4, 1, 5)
    per = float(statistics.median(secs))
    return {"value": 4.0 * (rows * 8192 + 8192 + rows) / per / 1e9, "unit": "GB/s",
            "cores": cores, "kind": "reference",
            "sample": f"{rows} of 65536 rows of A, median of 5 gemv calls, {per * 1e3:.1f} ms each"}


def run_reference_arm(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    if args.workload != "c2":
        emit({"impl": "reference", "unavailable": f"reference arm is implemented for the c2 "
              f"workload (the headline); {args.workload} was asked"})
        return 0
    from oracle import oracle as O

    if O.reference() is None:
        emit({"impl": "reference", "unavailable": "oracle/_ref/libmfref.so (the reference built "
              "from its sources) is not present on this machine"})
        return 0

    n = k = 8192
    ref = O.reference()
    ref.mfref_set_threads(host_threads())
    cores = int(ref.mfref_max_threads())
    # each step is the whole C2 problem (one 8192-row block; ~0.8 s on 16 host threads), on
    # inputs the reference's own Philox factories made once
    bench = O.RefGemmBench(8192, n, k, True, 1)
    # warm-up calls: as asked, up to three (a CPU call has nothing left to warm after one)
    warm_run = max(1, min(args.warmup, 3)) if args.warmup else 0
    if warm_run:
        bench.run(0.5, 1.0, True, warm_run)
    secs = list(bench.run(0.5, 1.0, True, args.steps))
    bench.close()
    per = statistics.median(secs)
    flops = 2.0 * 8192 * n * k
    value = flops / per / 1e12
    emit({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (the reference's Philox normal/uniform)",
        "config": {"workload": "C2: fused gemm C = 0.5*A@B^T + 1.0*C_in + bias, M=8192 N=8192 "
                               "K=8192 per rank (the reference's public gemm + bias_add on the "
                               "host CPU; at N > 1 GPUs the CPU's throughput is that of one "
                               "8192-row block, whatever the number of blocks)",
                   "precision": "fp32 (the reference's CPU packed GEMM)",
                   "m_per_rank": 8192, "n": n, "k": k, "same_config": True},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                         "sample": f"the whole C2 problem (all 8192 rows), median of "
                                   f"{len(secs)} timed calls after {warm_run} warm-up calls, "
                                   f"{per:.2f} s each"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })
    return 0


# ---- legs reported beside the main line ------------------------------------------------------

def time_back_to_back(step, seconds, ms_hint, stream, barrier, max_over_ranks, gpu_index):
    """Steps run back to back for about `seconds` of device time (so the GPU settles under its
    power cap), with their own clock record. Returns the sub-object of the JSON line."""
    from mensurflow_b200 import _lib
    import torch

    n = max(10, int(seconds * 1e3 / max(ms_hint, 1e-3)) + 1)
    clocks = ClockSampler(gpu_index)
    clocks.start()
    time.sleep(0.25)
    _lib.kernel_timer(True)
    _lib.kernel_timer_read()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    kern_ms, _ = _lib.kernel_timer_read()
    _lib.kernel_timer(False)
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    kern = max_over_ranks(kern_ms / n)
    return {"steps": n, "seconds": ms * n / 1e3, "ms_per_step": ms, "kernel_ms_per_step": kern,
            "clocks": clk}


def c5_strong_scaling(args, world, rank, device, gen, barrier, max_over_ranks, stream, peaks,
                      dist):
    """C5: 32768 x 32768 x 8192, alpha 1, beta 0, A and B uniform
    [-1, 1), rows of A and C split over the ranks with B replicated (strong scaling: the total work
    is fixed). Each rank writes its own slice; the gather of C to rank 0 is timed apart, both as
    NCCL's all_gather_into_tensor and fused into the GEMM (each rank's epilogue stores its rows
    into rank 0's buffer over NVLink)."""
    import mensurflow_b200 as mf
    from mensurflow_b200 import _lib
    import torch

    m_total, n, k = 32768, 32768, 8192
    m = m_total // world
    A = torch.rand(m, k, device=device, generator=gen) * 2 - 1
    B = torch.rand(k, n, device=device, generator=gen) * 2 - 1
    out = torch.empty(m, n, device=device)
    flops = 2.0 * m_total * n * k

    def step():
        mf.gemm(A, B, 1.0, None, 0.0, out=out, precision=args.precision)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.25)
    _lib.kernel_timer(True)
    _lib.kernel_timer_read()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.c5_steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    kern_ms, _ = _lib.kernel_timer_read()
    _lib.kernel_timer(False)
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.c5_steps)
    kern = max_over_ranks(kern_ms / args.c5_steps)
    per_product = 3.0 if args.precision == "3xtf32" else 1.0
    peak = peaks["bf16_burst"] / 2.0 / per_product
    res = {"workload": "C5: gemm 32768x32768x8192, alpha=1 beta=0, uniform[-1,1) inputs, rows "
                       "of A and C split over the ranks, B replicated (strong scaling)",
           "m_per_rank": m, "n": n, "k": k, "steps": args.c5_steps, "ms_per_step": ms,
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "scaling": "strong",
           "kernel_ms_per_step": kern,
           "per_gpu_kernel_frac": (flops / world) / (kern * 1e-3) / 1e12 / peak,
           "clocks": clk, "parallelism": f"dp{world} row blocks, each rank writes its own slice"}
    if world > 1:
        from mensurflow_b200 import sharded

        def t_steps(fn, reps=5):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            barrier()
            h0 = torch.cuda.Event(enable_timing=True)
            h1 = torch.cuda.Event(enable_timing=True)
            h0.record(stream)
            for _ in range(reps):
                fn()
            h1.record(stream)
            torch.cuda.synchronize()
            return max_over_ranks(h0.elapsed_time(h1) / reps)

        g_ms = t_steps(lambda: sharded.gather_rows(out, m_total))
        peer = sharded.PeerRowGather(m_total, n, device, root=0)
        flag = torch.zeros(1, device=device)

        def fused_step():
            sharded.gemm_into_peer(A, B, 1.0, None, 0.0, False, peer.row_ptr(rank * m), n,
                                   precision=args.precision, peer_memory=rank != 0)
            dist.all_reduce(flag)

        def barrier_step():
            step()
            dist.all_reduce(flag)

        f_runs, b_runs = [], []
        for _ in range(2):  # alternated, so clock drift under the power cap hits both alike
            f_runs.append(t_steps(fused_step))
            b_runs.append(t_steps(barrier_step))
        f_ms, b_ms = min(f_runs), min(b_runs)
        peer.close()
        into_root = 4.0 * (m_total - m) * n
        res.update({
            "nccl_all_gather_ms": g_ms,
            "nccl_all_gather_what": "NCCL all_gather_into_tensor of the C row blocks, alone",
            "gathered": {
                "ms_per_step": f_ms, "value": flops / (f_ms * 1e-3) / 1e12,
                "gemm_with_step_barrier_ms": b_ms,
                "bytes_into_rank0_per_step": into_root,
                "gbs_into_rank0": into_root / (f_ms * 1e-3) / 1e9,
                "what": "each rank's GEMM epilogue stores its rows into rank 0's C over NVLink "
                        "(CUDA IPC mapping), then a 1-element all_reduce as the step barrier; "
                        "rank 0 then holds the whole C"}})
    del A, B, out
    torch.cuda.empty_cache()
    return res


# ---- my arm -----------------------------------------------------------------------------------

def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    import mensurflow_b200 as mf
    from mensurflow_b200 import _lib

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peaks = load_peaks()
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    warm = max(3, args.warmup)

    e2e_factory = None
    gather_step = None
    fused_factory = None
    if args.workload in ("c2", "c5"):
        if args.workload == "c2":
            m = n = k = args.size               # per rank: weak scaling
            if args.mnk:
                m, n, k = (int(v) for v in args.mnk.split(","))
            scaling = "weak"
            alpha, beta, use_bias, trans_b = 0.5, 1.0, True, True
            wl = (f"C2: fused gemm C = 0.5*A@B^T + 1.0*C_in + bias, M={m} N={n} K={k} per rank "
                  f"(row block of an M={m}*N problem, B replicated)")
        else:
            m_total, n, k = 32768, 32768, 8192  # strong scaling: rows split over ranks
            if m_total % world:
                raise SystemExit("c5: world size must divide 32768")
            m = m_total // world
            scaling = "strong"
            alpha, beta, use_bias, trans_b = 1.0, 0.0, False, False
            wl = "C5: gemm 32768x32768x8192, alpha=1 beta=0, rows split over ranks"
        A = torch.randn(m, k, device=device, generator=gen)
        B = torch.randn(n, k, device=device, generator=gen) if trans_b else \
            torch.rand(k, n, device=device, generator=gen) * 2 - 1
        if args.workload == "c5":
            A.uniform_(-1, 1, generator=gen)
        C_in = torch.randn(m, n, device=device, generator=gen) if beta != 0 else None
        bias = (torch.rand(n, device=device, generator=gen) * 0.2 - 0.1) if use_bias else None
        out = torch.empty(m, n, device=device)
        flops_rank = 2.0 * m * n * k

        def step():
            mf.gemm(A, B, alpha, C_in, beta, False, trans_b, bias=bias, out=out,
                    precision=args.precision)

        if args.workload == "c5" and world > 1:
            from mensurflow_b200 import sharded

            def gather_step():
                return sharded.gather_rows(out, m * world)

            def fused_factory():
                # the GEMM whose epilogue stores every rank's rows into rank 0's C over NVLink,
                # then the step barrier; returns (step, cleanup)
                peer = sharded.PeerRowGather(m * world, n, device, root=0)
                flag = torch.zeros(1, device=device)

                def fused_step():
                    sharded.gemm_into_peer(A, B, alpha, C_in, beta, trans_b,
                                           peer.row_ptr(rank * m), n, bias=bias,
                                           precision=args.precision, peer_memory=rank != 0)
                    dist.all_reduce(flag)

                def barrier_step():
                    # the same step with each rank writing its own rows: the fused gather's
                    # cost is the difference
                    step()
                    dist.all_reduce(flag)
                return fused_step, barrier_step, peer.close

        unit = "TFLOP/s"
        h2d_bytes = 4 * (A.numel() + B.numel() + (C_in.numel() if C_in is not None else 0) +
                         (n if use_bias else 0))
        d2h_bytes = 4 * out.numel()

        def e2e_factory():
            hA = A.cpu().pin_memory()
            hB = B.cpu().pin_memory()
            hC = C_in.cpu().pin_memory() if C_in is not None else None
            hbias = bias.cpu().pin_memory() if bias is not None else None
            hout = torch.empty(m, n, pin_memory=True)

            def e2e_step():
                # the public op on host tensors with execution="gpu": inputs copied in, result
                # copied back (pipelined by row blocks), all inside the timed region
                mf.gemm(hA, hB, alpha, hC, beta, False, trans_b, bias=hbias, out=hout,
                        precision=args.precision, execution="gpu")
            return e2e_step
    elif args.workload == "c3":
        rows, d_in, d_hid = 4096, 1024, 4096    # per rank: weak scaling
        m, n, k = rows, d_in, d_hid
        scaling = "weak"
        wl = ("C3: MLP forward Y = gelu(X@W1 + b1)@W2 + b2, X [4096,1024], W1 [1024,4096], "
              "W2 [4096,1024], two fused gemm calls (bias + exact GELU in the epilogue)")
        X = torch.randn(rows, d_in, device=device, generator=gen)
        lim = (6.0 / (d_in + d_hid)) ** 0.5
        W1 = (torch.rand(d_in, d_hid, device=device, generator=gen) * 2 - 1) * lim
        W2 = (torch.rand(d_hid, d_in, device=device, generator=gen) * 2 - 1) * lim
        b1 = torch.zeros(d_hid, device=device)
        b2 = torch.zeros(d_in, device=device)
        flops_rank = 2.0 * rows * d_in * d_hid * 2
        unit = "TFLOP/s"
        h2d_bytes = 4 * (X.numel() + W1.numel() + W2.numel() + d_hid + d_in)
        d2h_bytes = 4 * rows * d_in
        W1_dense, W2_dense = W1, W2

        def mlp_by_row_blocks(hx, dx, dmid, dy, hy, w1, w2, bias1, bias2, s_in, s_out,
                              blocks=4):
            """Y = gelu(X W1 + b1) W2 + b2 from pinned host X into pinned host Y. A row of Y
            needs only its row of X, so block j's rows of X come in on s_in, both layers run on
            the caller's stream and its rows of Y go back on s_out: the copies of one block
            overlap the math of another. w1, w2: PackedB."""
            step_rows = rows // blocks
            for j in range(blocks):
                r0, r1 = j * step_rows, (j + 1) * step_rows
                with torch.cuda.stream(s_in):
                    dx[r0:r1].copy_(hx[r0:r1], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(s_in)
                stream.wait_event(ready)
                mf.gemm_prepacked(dx[r0:r1], w1, bias=bias1, activation="gelu",
                                  out=dmid[r0:r1])
                mf.gemm_prepacked(dmid[r0:r1], w2, bias=bias2, out=dy[r0:r1])
                done = torch.cuda.Event()
                done.record(stream)
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    hy[r0:r1].copy_(dy[r0:r1], non_blocking=True)
            stream.wait_stream(s_out)

        def e2e_factory():
            # the forward from pinned host tensors: weights and inputs copied in every step, the
            # output copied back, all inside the timed region. W1 and the biases cross first,
            # then X's first row block, then W2, then X's other blocks, so the first block's
            # layer 1 runs while W2 crosses; each weight is split once, as soon as it has landed.
            # Three blocks, the last the smallest (3/8, 3/8, 1/4 of the rows): measured 1.36 ms
            # per step against 1.41 for four equal blocks with both weights first (one box).
            hs = [t.cpu().pin_memory() for t in (X, W1_dense, W2_dense, b1, b2)]
            ds = [torch.empty_like(t) for t in (X, W1_dense, W2_dense, b1, b2)]
            dmid = torch.empty(rows, d_hid, device=device)
            dy = torch.empty(rows, d_in, device=device)
            hy = torch.empty(rows, d_in, pin_memory=True)
            s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
            bounds = (0, 3 * rows // 8, 6 * rows // 8, rows)

            def e2e_step():
                s_in.wait_stream(stream)
                x_in = []
                with torch.cuda.stream(s_in):
                    for i in (1, 3, 4):
                        ds[i].copy_(hs[i], non_blocking=True)
                    w1_in = torch.cuda.Event()
                    w1_in.record(s_in)
                    for j in range(len(bounds) - 1):
                        r0, r1 = bounds[j], bounds[j + 1]
                        ds[0][r0:r1].copy_(hs[0][r0:r1], non_blocking=True)
                        x_in.append(torch.cuda.Event())
                        x_in[-1].record(s_in)
                        if j == 0:
                            ds[2].copy_(hs[2], non_blocking=True)
                            w2_in = torch.cuda.Event()
                            w2_in.record(s_in)
                stream.wait_event(w1_in)
                w1 = mf.pack_b(ds[1], precision=args.precision)
                w2 = None
                for j in range(len(bounds) - 1):
                    r0, r1 = bounds[j], bounds[j + 1]
                    stream.wait_event(x_in[j])
                    mf.gemm_prepacked(ds[0][r0:r1], w1, bias=ds[3], activation="gelu",
                                      out=dmid[r0:r1])
                    if w2 is None:
                        stream.wait_event(w2_in)
                        w2 = mf.pack_b(ds[2], precision=args.precision)
                    mf.gemm_prepacked(dmid[r0:r1], w2, bias=ds[4], out=dy[r0:r1])
                    done = torch.cuda.Event()
                    done.record(stream)
                    s_out.wait_event(done)
                    with torch.cuda.stream(s_out):
                        hy[r0:r1].copy_(dy[r0:r1], non_blocking=True)
                stream.wait_stream(s_out)
                torch.cuda.current_stream().synchronize()
                w1.free()
                w2.free()
            return e2e_step

        if args.prepacked:
            wl += "; W1, W2 pre-split once (pack_b) outside the timed region"
            W1 = mf.pack_b(W1, precision=args.precision)
            W2 = mf.pack_b(W2, precision=args.precision)
            # inference with the split weights resident: only X comes in and Y goes out
            h2d_bytes = 4 * X.numel()
            packed1, packed2 = W1, W2

            def e2e_factory():
                hx = X.cpu().pin_memory()
                dx = torch.empty_like(X)
                dmid = torch.empty(rows, d_hid, device=device)
                dy = torch.empty(rows, d_in, device=device)
                hy = torch.empty(rows, d_in, pin_memory=True)
                s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)

                def e2e_step():
                    s_in.wait_stream(stream)
                    mlp_by_row_blocks(hx, dx, dmid, dy, hy, packed1, packed2, b1, b2, s_in,
                                      s_out)
                return e2e_step

        def step():
            h = mf.linear(X, W1, b1, "gelu", precision=args.precision)
            mf.linear(h, W2, b2, precision=args.precision)
    elif args.workload == "c4":
        heads_total, seq, dh = args.heads, 2048, 128
        if heads_total % world:
            raise SystemExit("c4: world size must divide the number of heads")
        bh = heads_total // world                # batch x heads split over ranks
        m, n, k = seq, seq, dh
        scaling = "strong"
        scale = float(1.0 / dh ** 0.5)
        std = 1.0 / dh ** 0.5
        Q = torch.randn(bh, seq, dh, device=device, generator=gen) * std
        K = torch.randn(bh, seq, dh, device=device, generator=gen) * std
        V = torch.randn(bh, seq, dh, device=device, generator=gen) * std
        # the config counts both GEMMs dense (the reference computes every score); the causal
        # one-kernel path skips the 128-key tiles above the diagonal of each 256-query block
        flops_rank = 2.0 * (2.0 * bh * seq * seq * dh)
        tiles = sum(-(-min(seq, (qb + 1) * 256) // 128) for qb in range(-(-seq // 256)))
        executed_rank = 2.0 * 2.0 * bh * 256 * 128 * dh * tiles
        if args.c4_unfused:
            wl = (f"C4: attention GEMMs S = Q@K^T/sqrt(128) and O = P@V, batch*heads="
                  f"{heads_total} split over ranks ({bh} per rank), seq 2048, head_dim 128; P is a "
                  f"stand-in of S's shape (softmax is not on the timed path)")
            P = torch.softmax(torch.randn(bh, seq, seq, device=device, generator=gen), -1)
            executed_rank = flops_rank
        else:
            wl = (f"C4: causal attention O = softmax(Q@K^T/sqrt(128), causal) @ V in one kernel "
                  f"(3xTF32), batch*heads={heads_total} split over ranks ({bh} per rank), seq "
                  f"2048, head_dim 128; value counts the config's dense flops of both GEMMs")
        unit = "TFLOP/s"
        h2d_bytes = 4 * 3 * bh * seq * dh
        d2h_bytes = 4 * bh * seq * dh

        def e2e_factory():
            # the whole attention op of the reference's API (S = QK^T/sqrt(d), causal masked
            # softmax, O = PV) on pinned host q, k, v with execution="gpu": batch chunks stream
            # in, are attended and stream back, overlapped
            hq, hk, hv = (t.cpu().pin_memory() for t in (Q, K, V))
            ho = torch.empty(bh, seq, dh, pin_memory=True)

            def e2e_step():
                mf.attention(hq, hk, hv, causal=True, precision=args.precision,
                             execution="gpu", out=ho)
            return e2e_step

        def step():
            if args.c4_unfused:
                mf.gemm_strided_batched(Q, K, scale, None, 0.0, False, True,
                                        precision=args.precision)
                mf.gemm_strided_batched(P, V, precision=args.precision)
            else:
                mf.attention(Q, K, V, causal=True, scale=scale, precision=args.precision)
    elif args.workload == "copy":
        # Tensor::contiguous() of C2's transposed operand: what the unpatched reference does to
        # B^T before every CUDA gemm with transB (through the host, src/core/tensor.cpp:224-229)
        m = n = args.size
        k = 1
        scaling = "weak"
        if args.view == "transpose":
            wl = (f"copy: Tensor::contiguous() of an {m}x{n} transposed fp32 view (C2's B^T) on "
                  f"the device")
            Bsrc = torch.randn(n, m, device=device, generator=gen)
            view = Bsrc.t()
        elif args.view == "slice":
            wl = f"copy: Tensor::contiguous() of columns 4..{n + 3} of an {m}x{n + 8} fp32 matrix"
            Bsrc = torch.randn(m, n + 8, device=device, generator=gen)
            view = Bsrc[:, 4:n + 4]
        else:
            wl = f"copy: Tensor::contiguous() of every other column of an {m}x{2 * n} fp32 matrix"
            Bsrc = torch.randn(m, 2 * n, device=device, generator=gen)
            view = Bsrc[:, ::2]
        flops_rank = 0.0
        unit = "GB/s"
        h2d_bytes = 4 * Bsrc.numel()
        d2h_bytes = 4 * m * n

        def step():
            mf.contiguous(view)

        def e2e_factory():
            hB = Bsrc.cpu().pin_memory()
            hout = torch.empty(m, n, pin_memory=True)
            dB = torch.empty_like(Bsrc)

            def e2e_step():
                dB.copy_(hB, non_blocking=True)
                dview = dB.as_strided(view.shape, view.stride(), view.storage_offset())
                hout.copy_(mf.contiguous(dview), non_blocking=True)
            return e2e_step
    else:
        m, k = 65536, 8192
        if args.mnk:
            m, _, k = (int(v) for v in args.mnk.split(","))
        n = 1
        scaling = "weak"
        wl = f"gemv: y = A x, A [{m}, {k}] per rank, x [{k}], double accumulation"
        A = torch.rand(m, k, device=device, generator=gen) * 2 - 1
        x = torch.rand(k, device=device, generator=gen) * 2 - 1
        flops_rank = 2.0 * m * k
        unit = "GB/s"
        h2d_bytes = 4 * (A.numel() + k)
        d2h_bytes = 4 * m

        def step():
            mf.matvec(A, x)

        def e2e_factory():
            hA = A.cpu().pin_memory()
            hx = x.cpu().pin_memory()
            hy = torch.empty(m, pin_memory=True)
            dA, dx = torch.empty_like(A), torch.empty_like(x)

            def e2e_step():
                dA.copy_(hA, non_blocking=True)
                dx.copy_(hx, non_blocking=True)
                hy.copy_(mf.matvec(dA, dx), non_blocking=True)
            return e2e_step

    # C3's operands (16-64 MiB) fit in L2: flush it between timed steps with this buffer
    flush_l2 = (torch.empty(64 << 20, device=device) if args.workload == "c3" else None)
    l2_note = ("L2 flushed between timed steps (256 MiB written, outside the timed intervals)"
               if flush_l2 is not None else "inputs larger than L2 (each operand >= 256 MiB)")

    # warm-up
    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    assert mf.device_status() == 0, "a kernel recorded a fault during warm-up"

    # timed region (device time, max over ranks)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    _lib.kernel_timer(True)
    _lib.kernel_timer_read()
    launches0 = _lib.launch_count()
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    if flush_l2 is None:
        # every step's operands are larger than L2: the steps run back to back
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
    else:
        # operands smaller than L2: each step timed alone, with L2 flushed (a buffer larger than
        # L2 written) between steps, outside the timed intervals
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for a, b in evs:
            flush_l2.zero_()
            a.record(stream)
            step()
            b.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = _lib.launch_count() - launches0
    kern_ms, kern_n = _lib.kernel_timer_read()
    _lib.kernel_timer(False)
    clk = clocks.stop()
    if flush_l2 is None:
        ms_local = e0.elapsed_time(e1) / args.steps
    else:
        ms_local = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    ms = max_over_ranks(ms_local)
    # device time of the tensor-core (or gemv) kernels per step, max over ranks
    kern_step_ms = max_over_ranks(kern_ms / args.steps)
    kern_per_step = kern_n / args.steps
    assert mf.device_status() == 0, "a kernel recorded a fault during the timed region"

    if args.workload == "copy":
        bytes_rank = 8.0 * m * n  # each element read once and written once
        value = world * bytes_rank / (ms * 1e-3) / 1e9
        achieved = bytes_rank / (kern_step_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": profiled_traffic("copy", "f32"),
                    "peak_source": f"{peaks['source']} hbm_gbs (STREAM-style copy)",
                    "kernel": {"transpose": "copy_transpose_kernel"}.get(
                        args.view, "copy_rows_kernel"),
                    "algorithmic_bytes_per_launch": bytes_rank}
    elif args.workload == "gemv":
        bytes_rank = 4.0 * (m * k + k + m)
        value = world * bytes_rank / (ms * 1e-3) / 1e9
        achieved = bytes_rank / (kern_step_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": profiled_traffic("gemv", "f64acc"),
                    "peak_source": f"{peaks['source']} hbm_gbs (STREAM-style copy)",
                    "algorithmic_bytes_per_launch": bytes_rank}
    else:
        value = world * flops_rank / (ms * 1e-3) / 1e12
        # the kernel's own work: equal to the config's flops except for the causal one-kernel
        # attention, which skips the masked tiles
        work = executed_rank if args.workload == "c4" else flops_rank
        achieved = work / (kern_step_ms * 1e-3) / 1e12
        per_product = 3.0 if args.precision == "3xtf32" else 1.0
        # tcgen05 kind::tf32 runs at half the kind::f16 rate; 3xTF32 issues three MMAs per term.
        # The kernel is timed in a sub-second burst at full clocks, so the burst figure is the
        # denominator; the sustained (power-capped) one is reported beside it.
        peak = peaks["bf16_burst"] / 2.0 / per_product
        peak_sustained = peaks["bf16_sustained"] / 2.0 / per_product
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "frac_of_sustained_peak": achieved / peak_sustained,
                    "traffic": profiled_traffic("c4unfused" if args.workload == "c4" and
                                                args.c4_unfused else args.workload,
                                                args.precision),
                    "peak_source": (f"{peaks['source']} bf16 burst {peaks['bf16_burst']} "
                                    f"TFLOP/s / 2 (TF32) / {int(per_product)} "
                                    f"({args.precision})"),
                    "kernel": "gemm_tc_kernel", "kernel_ms_per_step": kern_step_ms,
                    "kernel_launches_per_step": kern_per_step,
                    "algorithmic_flops_per_step": work}
        if args.workload == "c4" and not args.c4_unfused:
            roofline.update({
                "kernel": "attn_tc_kernel",
                "dense_equivalent_flops_per_step": flops_rank,
                "executed_value": world * executed_rank / (ms * 1e-3) / 1e12,
                "dense_equivalent_kernel_tflops": flops_rank / (kern_step_ms * 1e-3) / 1e12,
                "note": "achieved counts the flops the causal kernel executes (2 x 2 x 256 x 128 x "
                        "128 per visited key tile of a 256-query block); value counts the config's "
                        "dense flops of both GEMMs"})

    # end to end through the public API with host buffers (pinned), copies inside the timing
    e2e = None
    if args.e2e_steps > 0 and e2e_factory is not None:
        e2e_steps = min(args.e2e_steps, args.steps)
        e2e_step = e2e_factory()
        e2e_step()
        torch.cuda.synchronize()
        barrier()
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(f0.elapsed_time(f1) / e2e_steps)
        barrier()
        if args.workload in ("gemv", "copy"):
            e_val = world * bytes_rank / (e_ms * 1e-3) / 1e9
        else:
            e_val = world * flops_rank / (e_ms * 1e-3) / 1e12
        # this box's host link, for reading e2e: one pinned 256 MiB copy each way, and both at once
        hbuf = torch.empty(64 << 20, pin_memory=True)
        dbuf = torch.empty(64 << 20, device=device)
        link = {}
        for what in ("h2d", "d2h"):
            best = 0.0
            for _ in range(3):
                l0 = torch.cuda.Event(enable_timing=True)
                l1 = torch.cuda.Event(enable_timing=True)
                l0.record(stream)
                if what == "h2d":
                    dbuf.copy_(hbuf, non_blocking=True)
                else:
                    hbuf.copy_(dbuf, non_blocking=True)
                l1.record(stream)
                torch.cuda.synchronize()
                best = max(best, hbuf.numel() * 4 / (l0.elapsed_time(l1) * 1e-3) / 1e9)
            link[f"{what}_gbs"] = best
        # both directions at once (each on its own stream): on these boxes each runs ~10 %
        # slower than alone, which the simple bound below does not count
        hbuf2 = torch.empty(64 << 20, pin_memory=True)
        dbuf2 = torch.empty(64 << 20, device=device)
        s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        duplex = {"h2d_gbs": 0.0, "d2h_gbs": 0.0}
        for _ in range(3):
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            with torch.cuda.stream(s_h2d):
                ev[0].record(s_h2d)
                dbuf.copy_(hbuf, non_blocking=True)
                ev[1].record(s_h2d)
            with torch.cuda.stream(s_d2h):
                ev[2].record(s_d2h)
                hbuf2.copy_(dbuf2, non_blocking=True)
                ev[3].record(s_d2h)
            torch.cuda.synchronize()
            duplex["h2d_gbs"] = max(duplex["h2d_gbs"],
                                    hbuf.numel() * 4 / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9)
            duplex["d2h_gbs"] = max(duplex["d2h_gbs"],
                                    hbuf.numel() * 4 / (ev[2].elapsed_time(ev[3]) * 1e-3) / 1e9)
        link["both_directions"] = duplex
        del hbuf, dbuf, hbuf2, dbuf2
        bound_ms = max(h2d_bytes / (link["h2d_gbs"] * 1e9), d2h_bytes / (link["d2h_gbs"] * 1e9)) * 1e3
        # The same bound with the two directions slowing each other while both run: the smaller
        # direction overlaps the larger one completely, at the rates measured with both running,
        # and the rest of the larger one runs alone.
        hb, db = h2d_bytes / 1e9, d2h_bytes / 1e9
        if hb >= db:
            both_s = db / duplex["d2h_gbs"]
            duplex_ms = (both_s + max(0.0, hb - duplex["h2d_gbs"] * both_s) / link["h2d_gbs"]) * 1e3
        else:
            both_s = hb / duplex["h2d_gbs"]
            duplex_ms = (both_s + max(0.0, db - duplex["d2h_gbs"] * both_s) / link["d2h_gbs"]) * 1e3
        e2e = {"value": e_val, "unit": unit, "h2d_bytes_per_step": h2d_bytes,
               "d2h_bytes_per_step": d2h_bytes, "ms_per_step": e_ms, "steps": e2e_steps,
               "host_link": link, "link_bound_ms_per_step": bound_ms,
               "link_bound_both_directions_ms_per_step": duplex_ms,
               "path": E2E_PATHS.get(args.workload, E2E_PATHS["default"])}

    allgather = None
    if gather_step is not None:
        gather_step()
        torch.cuda.synchronize()
        barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(5):
            gather_step()
        g1.record(stream)
        torch.cuda.synchronize()
        g_ms = max_over_ranks(g0.elapsed_time(g1) / 5)
        allgather = {"ms": g_ms, "bytes_received_per_rank": 4 * m * n * (world - 1),
                     "what": "NCCL all_gather_into_tensor of the C row blocks (timed separately)"}
    if fused_factory is not None:
        fused_step, barrier_step, fused_close = fused_factory()

        def time_steps(fn, reps=5):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            barrier()
            h0 = torch.cuda.Event(enable_timing=True)
            h1 = torch.cuda.Event(enable_timing=True)
            h0.record(stream)
            for _ in range(reps):
                fn()
            h1.record(stream)
            torch.cuda.synchronize()
            return max_over_ranks(h0.elapsed_time(h1) / reps)

        # alternate the two so clock drift under the power cap hits both alike
        f_runs, b_runs = [], []
        for _ in range(2):
            f_runs.append(time_steps(fused_step))
            b_runs.append(time_steps(barrier_step))
        f_ms, b_ms = min(f_runs), min(b_runs)
        fused_close()
        allgather = dict(allgather or {})
        allgather.update({
            "fused_gemm_gather_ms": f_ms, "gemm_with_step_barrier_ms": b_ms, "gemm_only_ms": ms,
            "fused_value": world * flops_rank / (f_ms * 1e-3) / 1e12,
            "fused_what": "each rank's GEMM epilogue stores its rows into rank 0's C over NVLink "
                          "(CUDA IPC mapping), then a 1-element all_reduce as the step barrier; "
                          "rank 0 holds the whole C"})

    cpu_baseline = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "c2"
            and args.size == 8192 and not args.mnk):
        res = cpu_gemm_sample(8192, 8192, 8192, target_s=4.0, reps=3)
        if res is not None:
            secs, rows, kind, cores = res
            per = statistics.median(secs)
            cpu_baseline = {"value": 2.0 * rows * 8192 * 8192 / per / 1e12, "unit": "TFLOP/s",
                            "cores": cores, "kind": kind,
                            "sample": f"reference public gemm(+bias_add) on {rows} of 8192 rows "
                                      f"(B full), median of 3 timed calls, {per:.2f} s each"}

    if (rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "copy"
            and args.view == "transpose"):
        from oracle import oracle as O

        if O.reference() is not None:
            O.reference().mfref_set_threads(host_threads())
            secs = O.ref_time_transpose_contiguous(m, n, 1, 3)
            per = float(np.median(secs))
            cpu_baseline = {"value": 8.0 * m * n / per / 1e9, "unit": "GB/s",
                            "cores": int(O.reference().mfref_max_threads()), "kind": "reference",
                            "sample": f"reference Tensor::contiguous() of the {m}x{n} transpose "
                                      f"(cpu::transpose_f32), median of 3 calls, "
                                      f"{per * 1e3:.1f} ms each"}

    if (rank == 0 and world == 1 and not args.no_cpu_baseline and cpu_baseline is None
            and args.workload in ("c3", "c4", "c5", "gemv") and not args.mnk):
        cpu_baseline = reference_cpu_baseline(args, m, n, k)

    # the same step back to back for a few seconds: the figure under the power cap, against the
    # sustained GEMM peak
    sustained = None
    if args.sustained_s > 0 and args.workload == "c2" and not args.mnk and args.size == 8192:
        sustained = time_back_to_back(step, args.sustained_s, ms, stream, barrier,
                                      max_over_ranks, local)
        sus_achieved = flops_rank / (sustained["kernel_ms_per_step"] * 1e-3) / 1e12
        sustained.update({
            "value": world * flops_rank / (sustained["ms_per_step"] * 1e-3) / 1e12,
            "unit": unit, "kernel_achieved": sus_achieved,
            "frac_of_sustained_peak": sus_achieved / peak_sustained,
            "sustained_peak": peak_sustained,
            "peak_source": f"{peaks['source']} bf16 sustained {peaks['bf16_sustained']} "
                           f"TFLOP/s / 2 (TF32) / {int(per_product)} ({args.precision})"})

    # C5 strong scaling beside the C2 line (same line at every N, so the 1 -> 8 GPU scaling of
    # the sharded GEMM is read from SCALE's per-N `c5` objects)
    c5 = None
    if args.c5_steps > 0 and args.workload == "c2" and not args.mnk and args.size == 8192 \
            and 32768 % world == 0:
        c5 = c5_strong_scaling(args, world, rank, device, gen, barrier, max_over_ranks, stream,
                               peaks, dist)

    metric = {"gemv": "gemv HBM GB/s (65536x8192 fp32)",
              "copy": "strided copy GB/s (Tensor::contiguous of a transposed 8192^2 fp32 view)"}
    line = None
    if rank == 0:
        line = {
            "metric": metric.get(args.workload, METRIC),
            "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded torch randn / uniform with the configs' distributions)",
            "config": {"workload": wl, "precision": args.precision, "m_per_rank": m, "n": n,
                       "k": k, "parallelism": f"dp{world} row-block shards, no collective",
                       "l2": l2_note},
            "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu_baseline,
            "e2e": e2e, "clocks": clk, "allgather": allgather, "sustained": sustained, "c5": c5,
        }
    if world > 1:
        dist.destroy_process_group()
    # the JSON line last on stdout, after anything NCCL prints while the group shuts down
    if line is not None:
        emit(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
