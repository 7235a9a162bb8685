#!/usr/bin/env python
"""Headline benchmark: fp32-accurate (3xTF32) GEMM TFLOP/s on B200, BASELINE config 4 at 8192^3.

One "step" is one M = N = K = 8192 fp32 GEMM C = A.B (A, B ~ N(0,1)) in 3xTF32 mode through the
library's C ABI (nnb_sgemm: pack/split kernels + the tcgen05 GEMM kernel). With N GPUs
(torchrun, one rank per GPU) the 8192 rows of A are split into N contiguous bands, every rank
holds all of B, computes its band of C, and each rank's GEMM epilogue stores its band into GPU 0's C
through peer memory (`--gather nccl`: an NCCL gather after the GEMM instead) every step (total work
fixed: strong scaling). Inputs are 256 MiB per operand, larger than the 126 MB L2,
so no flush is needed between steps.

Keys beyond the base contract:
  roofline      the GEMM kernel's fp32-algorithmic TFLOP/s (2*M*N*K per launch / its average
                event-timed duration) against the 3xTF32 ceiling = measured dense bf16 burst peak
                / 2 (TF32 rate) / 3 (three MMAs per fp32 product) -- the timed loop is one kernel
                repeated for well under a second; the sustained-peak fraction is given beside it;
  cpu_baseline  the reference's own AVX2 sgemm (built from its sources into oracle/_ref) on all
                host cores, on a row band of the same problem sized to about 4 s per call (median
                of 3 calls);
  configs       configs 1, 2, 3 and 5, the TF32 mode and the size sweep, one small entry each.

Output: the full record on a line starting "detail: ", then the headline JSON line (last, short).
  e2e           the same GEMM through the public API from pinned host buffers: H2D of A (band)
                and B, the GEMM, D2H of C, every step; `pcie_floor` times the same copies alone.
`python bench.py --impl reference` times the reference's CPU sgemm alone (see run_reference).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import signal
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "nn-cpp_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "fp32-accurate GEMM TFLOP/s"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
CPU_SAMPLE_ROWS = 1024


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("nnb", "reference"), default="nnb")
    ap.add_argument("--size", type=int, default=8192, help="M = N = K")
    ap.add_argument("--mode", choices=("fp32x3", "tf32"), default="fp32x3")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--gather", choices=("peer", "nccl"), default="peer",
                    help="N>1 GEMM: bands stored into GPU 0's C by the GEMM epilogue (peer) or an NCCL gather after it")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip config 4's size sweep (small profiling runs)")
    ap.add_argument("--workload", choices=("all", "gemm", "transformer", "cnn", "attention", "next"), default="all",
                    help="one config alone, or all: the config 4 line with configs 2, 3 and 5 inside")
    ap.add_argument("--t-steps", type=int, default=10, help="timed transformer steps")
    ap.add_argument("--t-warmup", type=int, default=3)
    return ap.parse_args()


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {**FALLBACK_PEAKS, "bf16_tflops_sustained": None, "source": "fallback"}


def load_traffic(workload: str):
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary (or None)."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    d = json.loads(path.read_text())
    return d.get(workload)


class ClockSampler:
    """nvidia-smi sampled every 100 ms while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.send_signal(signal.SIGTERM)
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append({"sm": float(f[1]), "max": float(f[2]), "power": float(f[3]),
                             "hw_slowdown": f[5], "hw_thermal_slowdown": f[6],
                             "sw_thermal_slowdown": f[7], "sw_power_cap": f[8]})
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        peak_power = max(r["power"] for r in rows)
        loaded = [r for r in rows if r["power"] >= 0.5 * peak_power] or rows
        reasons = sorted({k for r in loaded for k in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                                      "sw_power_cap") if r[k].lower().startswith("active")})
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": reasons, "samples": len(loaded), "power_w_max": peak_power}


# ---------------------------------------------------------------------------------------------
# CPU side: the reference's own sgemm (oracle/_ref) or, if that was not built, the oracle port
# ---------------------------------------------------------------------------------------------

class CpuGemm:
    """The reference's own sgemm (oracle/_ref) on row bands of the size^3 problem.

    Inputs are drawn once (mt19937 N(0,1)); a sample is one call on a `rows` x size x size band.
    Without the reference build, the oracle's single-thread triple loop stands in ("port").
    """

    def __init__(self, size: int):
        import numpy as np
        from oracle import orc

        self.np, self.orc, self.size = np, orc, size
        self.ref = orc.ref()
        self.cores = os.cpu_count() or 1
        self.kind = "reference" if self.ref is not None else "port"
        if self.ref is not None:
            self.ref.ref_set_threads(self.cores)
            self.max_rows = size
        else:
            self.cores = 1
            self.max_rows = 64
        self.b = orc.normal(2, size * size)
        self.a = orc.normal(1, self.max_rows * size)
        self.c = np.empty(self.max_rows * size, np.float32)

    def time_band(self, rows: int, reps: int) -> float:
        """Median seconds of one rows x size x size product."""
        rows = max(1, min(rows, self.max_rows))
        o, n = self.orc, self.size
        if self.ref is not None:
            return self.ref.ref_time_sgemm(rows, n, n, o.ptr(self.a), o.ptr(self.b), o.ptr(self.c), reps)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            o.orc.orc_sgemm_f32(0, 0, rows, n, n, o.ptr(self.a), n, o.ptr(self.b), n, o.ptr(self.c), n, 0)
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    def rows_for(self, seconds: float) -> int:
        """Band height whose product takes about `seconds` (probed with a small band)."""
        probe = min(64, self.max_rows)
        t = self.time_band(probe, 1)
        rows = int(probe * seconds / max(t, 1e-6)) // 64 * 64
        return max(64 if self.ref is not None else 1, min(rows, self.max_rows))

    def describe(self, rows: int, reps: int) -> str:
        who = ("nn::kernels::sgemm (reference v2.0.0 built from its sources, AVX2/FMA)" if self.ref is not None
               else "the oracle's fp32 triple loop (reference build absent)")
        return (f"{who} on a {rows} x {self.size} x {self.size} row band of the {self.size}^3 problem, "
                f"{self.cores} threads, median of {reps}")


def cpu_baseline(size: int):
    """10-30 s of reference CPU work on the host cores (rank 0, N = 1 only)."""
    cg = CpuGemm(size)
    rows = cg.rows_for(4.0)
    reps = 3
    sec = cg.time_band(rows, reps)
    return {"value": 2.0 * rows * size * size / sec / 1e12, "unit": UNIT, "cores": cg.cores, "kind": cg.kind,
            "sample": cg.describe(rows, reps)}


def run_reference(args, rank: int):
    """--impl reference: the reference's CPU sgemm on the host cores, same metric and config.

    Each step is one row band of the size^3 product sized to about 0.2 s, so that
    warmup + steps stays within about a minute. Only rank 0 runs; other ranks exit at once.
    """
    if rank != 0:
        return
    size = args.size
    cg = CpuGemm(size)
    rows = cg.rows_for(0.2)
    for _ in range(args.warmup):
        cg.time_band(rows, 1)
    secs = [cg.time_band(rows, 1) for _ in range(args.steps)]
    sec = statistics.median(secs)
    value = 2.0 * rows * size * size / sec / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) from mt19937",
        "config": {"workload": f"config 4: square fp32 GEMM M=N=K={size}, each step a {rows}-row band",
                   "l2": "inputs larger than L2"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cg.cores, "kind": cg.kind,
                         "sample": cg.describe(rows, args.steps)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------

SWEEP_SIZES = (1024, 2048, 4096, 8192, 16384)


def run_gemm_sweep(rank: int, world: int, local_rank: int, reps: int = 5):
    """Config 4's sweep: M = N = K over SWEEP_SIZES in both math modes, A and B ~ N(0,1), the M rows
    cut into one band per rank whose GEMM epilogue stores into GPU 0's C through peer memory (N > 1).
    Per size and mode: whole-job TFLOP/s over `reps` timed calls after two untimed ones (x4 calls below
    4096), device events, max over ranks, and the per-GPU fraction of the measured ceiling (3xTF32:
    dense bf16 / 6, TF32: / 2; burst and sustained). A call is one nnb_sgemm (packs and the kernel)
    replayed from a CUDA graph, so the small sizes measure the GPU rather than host dispatch."""
    import torch
    import torch.distributed as dist

    import nnb
    from nnb.graph import GraphedStep
    from nnb.parallel import PeerBuffer, row_bands

    dev = torch.device("cuda", local_rank)
    peaks = load_peaks()
    burst = peaks["bf16_tflops"]
    sustained = peaks.get("bf16_tflops_sustained") or burst
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    results = []
    for size in SWEEP_SIZES:
        r0, r1 = row_bands(size, world)[rank]
        rows = r1 - r0
        gen = torch.Generator(device=dev)
        gen.manual_seed(3000 + size)
        b = torch.randn(size, size, device=dev, generator=gen)
        gen.manual_seed(4000 + size + rank)
        a = torch.randn(max(rows, 1), size, device=dev, generator=gen)
        peer = PeerBuffer((size, size), owner=0) if world > 1 else None
        c = torch.empty(size, size, device=dev) if peer is None else None
        c_out = c if peer is None else peer.ptr + r0 * size * 4
        for mode, name, div in ((nnb.MATH_FP32X3, "fp32x3", 6.0), (nnb.MATH_TF32, "tf32", 2.0)):
            def call():
                if rows:
                    nnb.sgemm(False, False, rows, size, size, a, size, b, size, c_out, size, False, math_mode=mode)

            n_calls = reps if size >= 4096 else 4 * reps
            graphed = GraphedStep(call)
            for _ in range(2):
                graphed()
            if world > 1:
                dist.barrier(device_ids=[local_rank])
            clocks = ClockSampler(local_rank) if size >= 8192 else None     # loops long enough to sample
            if clocks is not None:
                clocks.start()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(n_calls):
                graphed()
            e1.record()
            torch.cuda.synchronize()
            clk = clocks.stop() if clocks is not None else None
            del graphed
            t = torch.tensor([e0.elapsed_time(e1) / n_calls], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
            tf = 2.0 * size ** 3 / (ms * 1e-3) / 1e12
            results.append({"size": size, "mode": name, "ms_per_step": ms, "tflops": tf,
                            "frac_of_burst": tf / world / (burst / div),
                            "frac_of_sustained": tf / world / (sustained / div),
                            "clocks": None if clk is None else {k: clk[k] for k in ("sm_mhz", "reasons", "power_w_max")}})
        if nnb.device_error() != 0:
            raise SystemExit(f"device error in the sweep at {size}")
        if peer is not None:
            peer.close()              # unmapped on every rank before GPU 0 may free its C
        del a, b, c, peer
        torch.cuda.empty_cache()
    return {"what": "config 4 sweep, M = N = K, one nnb_sgemm per step"
                    + (f", {world} row bands stored into GPU 0's C by the epilogues" if world > 1 else ""),
            "unit": UNIT, "peak_source": peaks["source"], "results": results}


def run_nnb(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    import nnb

    from nnb.parallel import PeerBuffer, gather_rows, row_bands

    size = args.size
    mode = nnb.MATH_FP32X3 if args.mode == "fp32x3" else nnb.MATH_TF32
    bands = row_bands(size, world)
    rows = bands[rank][1] - bands[rank][0]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000)
    b = torch.randn(size, size, device=dev, generator=gen)
    gen.manual_seed(2000 + rank)
    a = torch.randn(rows, size, device=dev, generator=gen)
    c = torch.empty(rows, size, device=dev)
    peer = PeerBuffer((size, size), owner=0) if world > 1 and args.gather == "peer" else None
    c_out = c if peer is None else peer.ptr + bands[rank][0] * size * 4

    def gemm_local():
        nnb.sgemm(False, False, rows, size, size, a, size, b, size, c, size, False, math_mode=mode)

    def gemm():
        # with a peer buffer the epilogue stores this rank's tiles straight into GPU 0's C over NVLink
        nnb.sgemm(False, False, rows, size, size, a, size, b, size, c_out, size, False, math_mode=mode)

    def step():
        gemm()
        if world > 1 and peer is None:
            gather_rows(c, bands, dst=0)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if nnb.device_error() != 0:
        raise SystemExit("device error during warm-up")

    clocks = ClockSampler(local_rank)
    clocks.start()
    nnb.trace_reset()
    nnb.trace_enable(True)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    nnb.trace_enable(False)
    launches = nnb.launch_count()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    gemm_ms_total, gemm_launches = nnb.trace_query(nnb.TRACE_GEMM)
    pack_ms_total, _ = nnb.trace_query(nnb.TRACE_PACK)
    kernel_ms = gemm_ms_total / max(gemm_launches, 1)
    stats = torch.tensor([ms, kernel_ms, pack_ms_total / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_max, kernel_ms_max, pack_ms_max = stats.tolist()

    # compute-only timing (no gather): the GEMM step alone
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(min(args.steps, 50)):
        gemm()
    e1.record()
    torch.cuda.synchronize()
    comp = torch.tensor([e0.elapsed_time(e1) / min(args.steps, 50)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(comp, op=dist.ReduceOp.MAX)

    # the collective baseline at N > 1: the GEMM into a local band, then an NCCL gather to GPU 0
    nccl_gather = None
    if world > 1:
        for _ in range(3):                # first gathers set up NCCL's peer connections: untimed
            gemm_local()
            gather_rows(c, bands, dst=0)
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(min(args.steps, 50)):
            gemm_local()
            gather_rows(c, bands, dst=0)
        e1.record()
        torch.cuda.synchronize()
        ng = torch.tensor([e0.elapsed_time(e1) / min(args.steps, 50)], device=dev, dtype=torch.float64)
        dist.all_reduce(ng, op=dist.ReduceOp.MAX)
        nccl_gather = ng.item()

    # end to end through the public API from pinned host memory
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    c_h = torch.empty(rows, size).pin_memory()
    e2e_steps = max(1, args.e2e_steps)
    for _ in range(2):            # first calls allocate the entry's device buffers and streams: untimed
        nnb.sgemm_host(False, False, rows, size, size, a_h, size, b_h, size, c_h, size, False, math_mode=mode)
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(e2e_steps):
        # the drop-in for nn::kernels::sgemm on host buffers: B and row bands of A copied in, band
        # GEMMs overlapping the copies, bands of C copied back, all inside the call
        nnb.sgemm_host(False, False, rows, size, size, a_h, size, b_h, size, c_h, size, False, math_mode=mode,
                       blocking=False)
    e1.record()
    torch.cuda.synchronize()
    e2e = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    # the PCIe floor of e2e: the same bytes copied in (A, B) and out (C) and nothing else, the two
    # directions concurrent as inside the call (a_h and b_h hold a's and b's values: a no-op rewrite)
    c_dev = torch.empty(rows, size, device=dev)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def host_copies():
        cur = torch.cuda.current_stream()
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            b.copy_(b_h, non_blocking=True)
            a.copy_(a_h, non_blocking=True)
        with torch.cuda.stream(s_out):
            c_h.copy_(c_dev, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    host_copies()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(e2e_steps):
        host_copies()
    e1.record()
    torch.cuda.synchronize()
    pcie = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(pcie, op=dist.ReduceOp.MAX)
    del c_dev
    if peer is not None:
        peer.close()              # unmapped on every rank before GPU 0 may free its C

    # the plain-TF32 mode on the same operands, reported beside the 3xTF32 headline (N = 1)
    tf32_mode = None
    if world == 1 and mode == nnb.MATH_FP32X3:
        def gemm_tf32():
            nnb.sgemm(False, False, rows, size, size, a, size, b, size, c, size, False, math_mode=nnb.MATH_TF32)
        for _ in range(3):
            gemm_tf32()
        torch.cuda.synchronize()
        nnb.trace_reset()
        nnb.trace_enable(True)
        e0.record()
        for _ in range(50):
            gemm_tf32()
        e1.record()
        torch.cuda.synchronize()
        nnb.trace_enable(False)
        t_ms, t_n = nnb.trace_query(nnb.TRACE_GEMM)
        tf32_step = e0.elapsed_time(e1) / 50
        tf32_mode = {"value": 2.0 * rows * size * size / (tf32_step * 1e-3) / 1e12, "unit": UNIT,
                     "ms_per_step": tf32_step, "kernel_ms": t_ms / max(t_n, 1),
                     "kernel_tflops": 2.0 * rows * size * size / (t_ms / max(t_n, 1) * 1e-3) / 1e12}

    # cuBLAS TF32 on the same operands: a measured TF32 tensor-core reference point (rank 0, N = 1)
    cublas_tf32 = None
    if world == 1:
        torch.backends.cuda.matmul.allow_tf32 = True
        for _ in range(3):
            torch.matmul(a, b, out=c)
        e0.record()
        for _ in range(20):
            torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize()
        torch.backends.cuda.matmul.allow_tf32 = False
        cublas_tf32 = 2.0 * rows * size * size / (e0.elapsed_time(e1) / 20 * 1e-3) / 1e12

    del a, b, c, a_h, b_h, c_h
    torch.cuda.empty_cache()
    sweep = run_gemm_sweep(rank, world, local_rank) if args.gather == "peer" and not args.no_sweep else None

    transformer = None
    if args.workload == "all":
        transformer = run_transformer(args.t_steps, args.t_warmup, rank, world, local_rank)
        if world == 1:
            transformer["cnn"] = run_cnn(20, 3, local_rank)
            transformer["attention"] = run_attention(10, 3, local_rank)
            transformer["matmul512"] = run_matmul512(local_rank)
            transformer["next_rows"] = run_next_rows(local_rank, with_cpu=not args.no_cpu_baseline)
        else:
            transformer["attention"] = run_attention_sharded(10, 3, rank, world, local_rank)
    if rank != 0:
        return
    flops = 2.0 * size ** 3
    value = flops / (ms_max * 1e-3) / 1e12
    peaks = load_peaks()
    mmas = 3 if mode == nnb.MATH_FP32X3 else 1
    # The timed loop is one kernel repeated for well under a second, the burst case of the measured
    # peaks; the sustained (seconds-long, power-capped) figure is reported beside it.
    bf16_peak = peaks["bf16_tflops"]
    bf16_sustained = peaks["bf16_tflops_sustained"]
    peak_kind = "burst"
    peak = bf16_peak / 2.0 / mmas
    achieved = 2.0 * rows * size * size / (kernel_ms_max * 1e-3) / 1e12
    workload = f"gemm_{size}_{args.mode}"
    traffic = load_traffic(workload)
    if traffic is not None:
        traffic = traffic * (rows / size)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "tf32x3" if mode == nnb.MATH_FP32X3 else "tf32",
        "data": "synthetic N(0,1), fixed seeds",
        "config": {"workload": f"config 4: square fp32 GEMM M=N=K={size}, {args.mode}, "
                               f"M-row-block sharded over {world} GPU(s), C gathered to GPU 0",
                   "parallelism": f"m-rows x{world}", "l2": "inputs > L2 (256 MiB per operand), no flush",
                   "math_mode": args.mode},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "gemm_tc_kernel", "kernel_ms": kernel_ms_max,
                     "peak_basis": f"{peaks['source']} dense bf16 {peak_kind} {bf16_peak} TFLOP/s / 2 (TF32 rate)"
                                   f" / {mmas} (MMAs per fp32 product)",
                     "frac_of_sustained_peak": (achieved / (bf16_sustained / 2.0 / mmas)) if bf16_sustained else None,
                     "cublas_tf32_tflops": cublas_tf32},
        "pack_ms_per_step": pack_ms_max,
        "ms_per_step_compute_only": comp.item(),
        "sweep": sweep,
        "tf32_mode": None if tf32_mode is None else dict(tf32_mode, roofline={
            "bound": "tensor", "achieved": tf32_mode["kernel_tflops"], "peak": bf16_peak / 2.0, "unit": UNIT,
            "frac": tf32_mode["kernel_tflops"] / (bf16_peak / 2.0),
            "frac_of_sustained_peak": (tf32_mode["kernel_tflops"] / (bf16_sustained / 2.0)) if bf16_sustained else None,
            "peak_basis": f"{peaks['source']} dense bf16 {peak_kind} {bf16_peak} TFLOP/s / 2 (TF32 rate)",
            "cublas_tf32_tflops": cublas_tf32}),
        "gather": None if world == 1 else (
            "fused: each rank's GEMM epilogue stores its tiles into GPU 0's C through CUDA IPC peer memory"
            if peer is not None else "NCCL gather after the GEMM"),
        "gather_baseline": None if nccl_gather is None else {
            "what": "GEMM into a local band, then an NCCL gather to GPU 0", "ms_per_step": nccl_gather,
            "value": flops / (nccl_gather * 1e-3) / 1e12, "unit": UNIT},
        "e2e": {"value": flops / (e2e.item() * 1e-3) / 1e12, "unit": UNIT,
                "h2d_bytes_per_step": int((rows * size + size * size) * 4 * world),
                "d2h_bytes_per_step": int(rows * size * 4 * world),
                "api": "nnb_sgemm_host_async (host buffers, page-locked): copies in, banded GEMMs, copy back",
                "pcie_floor": {"what": "the same bytes copied in and out concurrently, no GEMM",
                               "ms_per_step": pcie.item(), "e2e_ms_per_step": e2e.item(),
                               "frac": pcie.item() / e2e.item()}},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if transformer is not None:
        for key in ("cnn", "attention", "matmul512", "next_rows"):
            if key in transformer:
                line[key] = transformer.pop(key)
        line["transformer"] = transformer
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(size)
        if args.workload == "all":
            line["cpu_baselines_other_configs"] = cpu_baselines()
    # The full record first, on a line that is not JSON by itself; then the headline JSON line, kept
    # short (rounded numbers, one small entry per config) so the whole of it fits a short log tail.
    print("detail: " + json.dumps(line), flush=True)
    print(headline_text(line), flush=True)


def _r(x, digits=4):
    """x rounded to `digits` significant figures (None and non-numbers unchanged)."""
    if isinstance(x, bool) or not isinstance(x, (int, float)):
        return x
    if x == 0 or x != x:
        return x
    from math import floor, log10
    return round(x, max(0, digits - 1 - int(floor(log10(abs(x))))))


def headline_text(line: dict) -> str:
    """The headline JSON line (compact separators)."""
    return json.dumps(headline(line), separators=(",", ":"))


def headline(line: dict) -> dict:
    """The contract's keys from the full record, with each other config reduced to its key numbers."""
    keep = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "gpu_launches")
    out = {k: _r(line[k]) for k in keep if k in line}
    out["config"] = line["config"]
    rl = line["roofline"]
    if isinstance(rl.get("traffic"), float):
        rl = dict(rl, traffic=int(rl["traffic"]))
    out["roofline"] = {k: _r(rl.get(k)) for k in ("bound", "achieved", "peak", "unit", "frac", "traffic", "kernel",
                                                  "frac_of_sustained_peak", "cublas_tf32_tflops")}
    if "cpu_baseline" in line:
        cb = line["cpu_baseline"]
        out["cpu_baseline"] = {"value": _r(cb["value"]), "unit": cb["unit"], "cores": cb["cores"], "kind": cb["kind"],
                               "sample": cb["sample"][:60]}
    e = line["e2e"]
    out["e2e"] = {"value": _r(e["value"]), "unit": e["unit"], "h2d_bytes_per_step": e["h2d_bytes_per_step"],
                  "d2h_bytes_per_step": e["d2h_bytes_per_step"]}
    if line.get("clocks"):
        c = line["clocks"]
        out["clocks"] = {"sm_mhz": c.get("sm_mhz"), "sm_max_mhz": c.get("sm_max_mhz"), "reasons": c.get("reasons")}
    cfg = {}
    if line.get("tf32_mode"):
        t = line["tf32_mode"]
        cfg["c4_tf32"] = {"tflops": _r(t["value"]), "kernel": _r(t["kernel_tflops"]),
                          "frac": _r(t["roofline"]["frac"], 3)}
    if line.get("sweep"):       # 3xTF32 sizes here; the TF32-mode sweep stays in the detail line
        cfg["c4_sweep_x3"] = {str(r["size"]): _r(r["tflops"], 3) for r in line["sweep"]["results"]
                              if r["mode"] == "fp32x3"}
    if line.get("matmul512"):
        cfg["c1_tflops"] = _r(line["matmul512"]["value"], 3)
    if line.get("cnn"):
        cfg["c2_ms"] = _r(line["cnn"]["value"], 3)
    if line.get("attention"):
        a = line["attention"]
        cfg["c3"] = {"ms": _r(a["value"], 3), "tflops": _r(a.get("algorithmic_tflops_causal"), 3)}
    if line.get("transformer"):
        t = line["transformer"]
        cfg["c5"] = {"tok_s": _r(t["value"], 4), "ms": _r(t["ms_per_step"], 4), "tflops": _r(t["algorithmic_tflops"], 3),
                     "e2e_tok_s": _r(t["e2e"]["value"], 4)}
    if line.get("cpu_baselines_other_configs") and "unavailable" not in line["cpu_baselines_other_configs"]:
        c = line["cpu_baselines_other_configs"]
        cfg["cpu"] = {"c1_tflops": _r(c.get("config1_matmul512_tflops"), 3), "c2_ms": _r(c.get("config2_cnn_ms_per_step"), 3),
                      "c3_ms": _r(c.get("config3_attention_ms_per_step"), 3),
                      "c5_tok_s": _r(c.get("config5_transformer_tokens_per_s"), 4)}
    if line.get("gather_baseline"):
        cfg["nccl_gather_tflops"] = _r(line["gather_baseline"]["value"], 4)
    out["configs"] = cfg
    return out


# ---------------------------------------------------------------------------------------------
# Config 5: transformer training step (tokens/s)
# ---------------------------------------------------------------------------------------------

T5 = dict(vocab_size=4096, dim=512, heads=8, layers=4, max_len=512, batch=64, seq=512)
# algorithmic work per step (causal-effective attention): 88.08 MFLOP/token of matmuls (forward +
# backward) and 6.30 MFLOP/token of attention over 32768 tokens
T5_FLOP_PER_STEP = 3.093e12


def run_transformer(steps: int, warmup: int, rank: int, world: int, local_rank: int, group=None):
    """One config-5 step = forward, sequence cross entropy, backward and AdamW on the global batch
    of 64 x 512 tokens, cut into 8 virtual shards spread over the ranks (nnb.train)."""
    import torch

    import nnb
    from nnb.nn import AdamW, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer

    dev = torch.device("cuda", local_rank)
    cfg = TransformerConfig(T5["vocab_size"], T5["dim"], T5["heads"], T5["layers"], T5["max_len"])
    model = Transformer(cfg, seed=0, device=dev)
    opt = AdamW(model.parameters(), lr=3e-4, weight_decay=1e-2)
    tr = ShardedTrainer(model, opt, shards=8, world=world, rank=rank, group=group)
    g = torch.Generator().manual_seed(11)
    ids_h = torch.randint(0, T5["vocab_size"], (T5["batch"], T5["seq"] + 1), generator=g)
    x_h = ids_h[:, :-1].contiguous().pin_memory()
    y_h = ids_h[:, 1:].contiguous().pin_memory()
    x_d, y_d = x_h.to(dev), y_h.to(dev)
    loss_h = torch.empty(1).pin_memory()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local_rank])

    for _ in range(warmup):
        tr.step(x_d, y_d)
    torch.cuda.synchronize()
    first_loss = float(tr.loss.cpu()[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # eager dispatch, for reference: every op launched from the host
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        tr.step(x_d, y_d)
    e1.record()
    torch.cuda.synchronize()
    eager = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
    # the step captured once into a CUDA graph (one more real step first) and replayed
    nnb.trace_reset()                       # zeroes the launch counter; the tracer stays off here
    graphed = tr.capture(x_d, y_d, warmup=1)
    per_step_launches = nnb.launch_count() // 2          # the warm-up step and the captured one
    for _ in range(2):                                   # first replays upload the graph: untimed
        graphed()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        graphed()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    launches = per_step_launches * steps
    ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
    # end to end: ids and targets from pinned host memory every step, the loss read back every step
    e0.record()
    for _ in range(steps):
        loss = graphed(x_h, y_h)                 # pinned host -> the graph's input buffers
        loss_h.copy_(loss, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
    loss_final = float(graphed.loss.cpu()[0])
    graphed.release()
    # per-kind device time from the library's event tracer, on separate (untimed) steps: the tracer
    # records two events around every launch, which costs host time
    traced = min(steps, 3)
    nnb.trace_reset()
    nnb.trace_enable(True)
    for _ in range(traced):
        tr.step(x_d, y_d)
    torch.cuda.synchronize()
    nnb.trace_enable(False)
    kinds = {name: nnb.trace_query(k) for name, k in (("gemm", nnb.TRACE_GEMM), ("pack", nnb.TRACE_PACK),
                                                      ("rowwise", nnb.TRACE_ROWWISE), ("attention", nnb.TRACE_ATTENTION),
                                                      ("aux", nnb.TRACE_AUX))}
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
        dist.all_reduce(eager, op=dist.ReduceOp.MAX)
    tokens = T5["batch"] * T5["seq"]
    ms_v = ms.item()
    return {
        "metric": "transformer train tokens/s", "value": tokens / (ms_v * 1e-3), "unit": "tokens/s",
        "ms_per_step": ms_v, "steps": steps, "warmup": warmup, "scaling": "strong",
        "config": {"workload": "config 5: 4 pre-LN blocks, d 512, 8 heads, FFN 2048 GELU, vocab 4096, seq 512, "
                               "global batch 64, sequence CE, AdamW 3e-4",
                   "parallelism": f"data parallel x{world}, 8 virtual shards, fixed-order gradient sum",
                   "dispatch": "the whole step (collectives included) captured once into a CUDA graph and replayed",
                   "math_mode": "fp32x3"},
        "algorithmic_tflops": T5_FLOP_PER_STEP / (ms_v * 1e-3) / 1e12,
        "eager_ms_per_step": eager.item(),
        "loss_after_warmup": first_loss, "loss_final": loss_final,
        "kernel_ms_per_step": {k: v[0] / traced for k, v in kinds.items()},
        "l2": "inputs larger than L2 (weights, optimizer state and activations are several GB per step)",
        "gpu_launches": int(launches),
        "e2e": {"value": tokens / (e2e.item() * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x_h.numel() * 8 * 2), "d2h_bytes_per_step": 4},
    }


# ---------------------------------------------------------------------------------------------
# Config 2 (CNN forward + backward) and config 3 (causal attention forward + backward)
# ---------------------------------------------------------------------------------------------

CNN_FLOP_PER_STEP = 1.60e9            # conv1 28.9 M + conv2 462.4 M + fc 51.6 M forward, ~2x that backward
ATTN_FLOP_PER_STEP = 6.468e9          # causal-effective forward + backward, B32 H8 T256 Dh64


def _time_steps(torch, fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_cnn(steps: int, warmup: int, local_rank: int):
    """Config 2: conv2d_relu 1->32, maxpool, conv2d_relu 32->64, maxpool, flatten, linear 3136->128,
    relu, linear 128->10, cross entropy; forward + backward on a batch of 64 (one GPU: replicas only)."""
    import numpy as np
    import torch

    import nnb
    import nnb.functional as F
    from nnb.autograd import Value
    from nnb.nn import Conv2d, Flatten, Linear, MaxPool2d, ReLU, Sequential

    dev = torch.device("cuda", local_rank)
    rng = np.random.default_rng(2)
    net = Sequential(Conv2d(1, 32, 3, 1, 1, rng, dev), ReLU(), MaxPool2d(2, 2), Conv2d(32, 64, 3, 1, 1, rng, dev),
                     ReLU(), MaxPool2d(2, 2), Flatten(), Linear(3136, 128, rng, dev), ReLU(), Linear(128, 10, rng, dev))
    g = torch.Generator().manual_seed(4)
    x = torch.rand(64, 1, 28, 28, generator=g).to(dev)
    y = torch.randint(0, 10, (64,), generator=g).to(dev)

    def step():
        net.zero_grad()
        loss = F.cross_entropy_loss(net(Value.leaf(x, False)), y)
        loss.backward()

    from nnb.graph import GraphedStep

    nnb.trace_reset()
    eager = _time_steps(torch, step, steps, warmup)
    launches = nnb.launch_count() / (steps + warmup)
    ms = _time_steps(torch, GraphedStep(step), steps, warmup)
    return {"metric": "CNN fwd+bwd ms/step", "value": ms, "unit": "ms", "higher_is_better": False,
            "config": {"workload": "config 2: CNN 1x28x28 batch 64, conv2d_relu x2, maxpool x2, linear x2, CE",
                       "dispatch": "CUDA graph replay of the whole step"},
            "eager_ms": eager, "algorithmic_gflops": CNN_FLOP_PER_STEP / (ms * 1e-3) / 1e9,
            "launches_per_step": launches}


def run_attention(steps: int, warmup: int, local_rank: int):
    """Config 3: causal attention forward + backward, q/k/v [32, 256, 512], 8 heads, N(0,1). The fused
    kernels (nnb_flash_attention_*) are the timed path; the composed path that keeps the
    probabilities (nnb_attention_*, the reference's structure) is timed beside it."""
    import torch

    import nnb

    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(6)
    N, T, D, H = 32, 256, 512, 8
    q, k, v, go = (torch.randn(N, T, D, device=dev, generator=g) for _ in range(4))
    out, probs = torch.empty(N, T, D, device=dev), torch.empty(N, H, T, T, device=dev)
    stats = torch.empty(N, H, T, 2, device=dev)
    dq, dk, dv = (torch.empty(N, T, D, device=dev) for _ in range(3))
    L = nnb.lib()

    def fused():
        s = torch.cuda.current_stream().cuda_stream
        nnb.check(L.nnb_flash_attention_fwd(s, N, T, T, D, H, q.data_ptr(), k.data_ptr(), v.data_ptr(), None, 1,
                                            out.data_ptr(), stats.data_ptr()))
        nnb.check(L.nnb_flash_attention_bwd(s, N, T, T, D, H, go.data_ptr(), q.data_ptr(), k.data_ptr(),
                                            v.data_ptr(), out.data_ptr(), stats.data_ptr(), None, 1, dq.data_ptr(), 1,
                                            dk.data_ptr(), 1, dv.data_ptr(), 1))

    def composed():
        s = torch.cuda.current_stream().cuda_stream
        nnb.check(L.nnb_attention_fwd(s, N, T, T, D, H, q.data_ptr(), k.data_ptr(), v.data_ptr(), None, 1,
                                      out.data_ptr(), probs.data_ptr()))
        nnb.check(L.nnb_attention_bwd(s, N, T, T, D, H, go.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                      probs.data_ptr(), None, 1, dq.data_ptr(), 1, dk.data_ptr(), 1, dv.data_ptr(), 1))

    from nnb.graph import GraphedStep

    eager = _time_steps(torch, fused, steps, warmup)
    ms = _time_steps(torch, GraphedStep(fused), steps, warmup)
    composed_ms = _time_steps(torch, GraphedStep(composed), steps, warmup)
    # per-kernel device time of the fused step
    nnb.trace_reset()
    nnb.trace_enable(True)
    for _ in range(5):
        fused()
    kernels = {}
    for name, kind in (("pack", nnb.TRACE_PACK), ("attention", nnb.TRACE_ATTENTION)):
        t, n = nnb.trace_query(kind)
        kernels[name] = {"ms": round(t / 5, 4), "launches": n // 5}
    nnb.trace_enable(False)
    return {"metric": "causal attention fwd+bwd ms/step", "value": ms, "unit": "ms", "higher_is_better": False,
            "config": {"workload": "config 3: B32 H8 T256 Dh64 causal, fwd + bwd", "dispatch": "CUDA graph replay",
                       "path": "fused (no probability matrix)"},
            "eager_ms": eager, "composed_path_ms": composed_ms, "kernels": kernels,
            "algorithmic_tflops_causal": ATTN_FLOP_PER_STEP / (ms * 1e-3) / 1e12}


def run_attention_sharded(steps: int, warmup: int, rank: int, world: int, local_rank: int):
    """Config 3 on N GPUs: the batch x head units split by samples (32 / N per GPU), O, dQ, dK and dV
    gathered on GPU 0 (nnb.parallel.ShardedAttention: the backward kernels store dQ / dK / dV there
    through peer memory, O goes by a peer copy overlapping the backward). Max over ranks."""
    import torch
    import torch.distributed as dist

    from nnb.parallel import ShardedAttention

    dev = torch.device("cuda", local_rank)
    N, T, D, H = 32, 256, 512, 8
    sa = ShardedAttention(N, T, D, H, causal=True)
    g = torch.Generator(device=dev).manual_seed(6 + rank)
    q, k, v, go = (torch.randn(max(sa.local, 1), T, D, device=dev, generator=g) for _ in range(4))
    for _ in range(warmup):
        sa.step(q, k, v, go)
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local_rank])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        sa.step(q, k, v, go)
    e1.record()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local_rank])
    ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    sa.close()
    return {"metric": "causal attention fwd+bwd ms/step", "value": ms.item(), "unit": "ms", "higher_is_better": False,
            "n_gpus": world, "scaling": "strong",
            "config": {"workload": "config 3: B32 H8 T256 Dh64 causal, fwd + bwd",
                       "parallelism": f"samples x{world} ({N // world} per GPU), O / dQ / dK / dV gathered on GPU 0 "
                                      "(backward epilogues store through peer memory; O by a peer copy)"},
            "algorithmic_tflops_causal": ATTN_FLOP_PER_STEP / (ms.item() * 1e-3) / 1e12}


def run_matmul512(local_rank: int):
    """Config 1: C = A.B, M = N = K = 512, A then B from U[-1, 1], through nn::matmul's counterpart
    nnb_matmul (launch-bound: one pack pair and one tensor-core launch)."""
    import ctypes

    import torch

    import nnb

    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.rand(512, 512, device=dev, generator=g) * 2 - 1
    b = torch.rand(512, 512, device=dev, generator=g) * 2 - 1
    c = torch.empty(512, 512, device=dev)
    sh = (ctypes.c_int64 * 2)(512, 512)
    osh, ond = (ctypes.c_int64 * 16)(), ctypes.c_int()
    L = nnb.lib()

    def step():
        nnb.check(L.nnb_matmul(torch.cuda.current_stream().cuda_stream, a.data_ptr(), sh, 2, b.data_ptr(), sh, 2, 0,
                               0, c.data_ptr(), osh, ctypes.byref(ond)))

    from nnb.graph import GraphedStep

    eager = _time_steps(torch, step, 200, 20)
    ms = _time_steps(torch, GraphedStep(step), 200, 20)
    return {"metric": "matmul 512^3 TFLOP/s", "value": 2 * 512 ** 3 / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "us_per_call": ms * 1e3, "eager_us_per_call": eager * 1e3,
            "config": {"workload": "config 1: nn::matmul 512^3 fp32 (3xTF32)", "dispatch": "CUDA graph replay"}}


def run_next_rows(local_rank: int, with_cpu: bool = True):
    """The rows built after the hot path, each timed on the GPU beside the reference's own CPU code on
    the same shapes (oracle/_ref, all host cores, bounded samples): attention with dropout active,
    the dropout stream, the DataLoader, checkpoints and the general (dilated, grouped) conv."""
    import ctypes
    import tempfile

    import numpy as np
    import torch

    import nnb
    import nnb.functional as F
    import nnb.random as nr
    from nnb.autograd import Value
    from nnb.graph import GraphedStep

    dev = torch.device("cuda", local_rank)
    L = nnb.lib()
    ref = None
    if with_cpu:
        from oracle import orc
        ref = orc.ref()
        if ref is not None:
            ref.ref_set_threads(os.cpu_count() or 1)
    cores = os.cpu_count() or 1
    out = {}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def events(fn, reps):
        fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    # -- attention with dropout active (config-3 shape, p = 0.1), mask drawn inside the step ----------
    N, T, D, H, p = 32, 256, 512, 8, 0.1
    g = torch.Generator(device=dev).manual_seed(7)
    q, k, v, go = (torch.randn(N, T, D, device=dev, generator=g) for _ in range(4))
    nr.manual_seed(1)
    state = nr.device_generator("dropout", dev)
    keep = torch.empty((N * H * T * T + 31) // 32, dtype=torch.int32, device=dev)
    o, probs, wts = torch.empty(N, T, D, device=dev), torch.empty(N, H, T, T, device=dev), torch.empty(N, H, T, T, device=dev)
    dq, dk, dv = (torch.empty(N, T, D, device=dev) for _ in range(3))

    def mask():
        nnb.check(L.nnb_dropout_mask(torch.cuda.current_stream().cuda_stream, state.data_ptr(), N * H * T * T,
                                     ctypes.c_float(p), keep.data_ptr()))

    def attn_drop():
        s = torch.cuda.current_stream().cuda_stream
        mask()
        nnb.check(L.nnb_attention_dropout_fwd(s, N, T, T, D, H, q.data_ptr(), k.data_ptr(), v.data_ptr(), None, 1,
                                              ctypes.c_float(p), keep.data_ptr(), o.data_ptr(), probs.data_ptr(),
                                              wts.data_ptr()))
        nnb.check(L.nnb_attention_dropout_bwd(s, N, T, T, D, H, go.data_ptr(), q.data_ptr(), k.data_ptr(),
                                              v.data_ptr(), probs.data_ptr(), wts.data_ptr(), ctypes.c_float(p),
                                              keep.data_ptr(), None, 1, dq.data_ptr(), 1, dk.data_ptr(), 1,
                                              dv.data_ptr(), 1))

    step_ms = events(GraphedStep(attn_drop), 5)
    mask_ms = events(mask, 5)
    draws = N * H * T * T
    row = {"metric": "attention with dropout fwd+bwd ms/step", "value": step_ms, "unit": "ms",
           "config": {"workload": "config-3 shape B32 H8 T256 Dh64 causal, dropout 0.1 on the weights (composed path)",
                      "dispatch": "CUDA graph replay"},
           "mask_ms": mask_ms,
           "dropout_stream": {"draws_per_s": draws / (mask_ms * 1e-3), "draws": draws,
                              "bound": "serial: one mt19937 stream per layer (the reference's draw order), one CTA"}}
    if ref is not None:
        qa, ka, va, ga = (x.cpu().numpy().ravel() for x in (q, k, v, go))
        oa, dqa, dka, dva = (np.zeros(N * T * D, np.float32) for _ in range(4))
        t0 = time.perf_counter()
        ref.ref_attention_dropout(1, N, T, D, H, 1, p, *(orc.ptr(a) for a in (qa, ka, va, ga, oa, dqa, dka, dva)))
        row["cpu_baseline"] = {"value": (time.perf_counter() - t0) * 1e3, "unit": "ms", "cores": cores,
                               "kind": "reference", "sample": "one full fwd+bwd of the same shape"}
        sizes = np.array([1 << 22], np.uintp)
        masks = np.zeros(1 << 22, np.float32)
        t0 = time.perf_counter()
        ref.ref_dropout_masks(1, 0, p, sizes.ctypes.data, 1, masks.ctypes.data)
        row["dropout_stream"]["cpu_baseline_draws_per_s"] = (1 << 22) / (time.perf_counter() - t0)
    out["attention_dropout"] = row

    # -- DataLoader: batches gathered from an HBM-resident dataset, and the host path -------------------
    from nnb.data import DataLoader, SequenceDataset, TensorDataset
    n, feat = 60000, 784
    xs = np.random.default_rng(0).random((n, 1, 28, 28), dtype=np.float32)
    ys = np.random.default_rng(1).integers(0, 10, n).astype(np.int64)
    nr.manual_seed(2)
    ld = DataLoader(TensorDataset(xs, ys), 64, True, device=dev)
    ld.get_batch(0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record()
    for xb, yb in ld:
        pass
    e1.record()
    torch.cuda.synchronize()
    epoch_s = time.perf_counter() - t0
    nb = ld.num_batches()
    big = DataLoader(TensorDataset(xs, ys), 8192, True, device=dev)
    big_ms = events(lambda: big.get_batch(1), 10)
    moved = 2 * 8192 * (feat * 4 + 8)
    seq = DataLoader(SequenceDataset(np.random.default_rng(3).integers(0, 4096, 1 << 24), 512), 64, True, device=dev)
    seq_ms = events(lambda: seq.get_batch(5), 20)
    row = {"metric": "DataLoader batch (64 x 1x28x28 + labels) us", "value": epoch_s / nb * 1e6, "unit": "us",
           "config": {"workload": "MNIST-shaped TensorDataset 60000 x 784 fp32 + int64 labels in HBM, batch 64, "
                                  "shuffled epoch (host wall time per batch, Python iteration included)"},
           "device_us_per_batch": e0.elapsed_time(e1) / nb * 1e3,
           "gather_8192": {"ms": big_ms, "gbs": moved / (big_ms * 1e-3) / 1e9,
                           "roofline": {"bound": "hbm", "achieved": moved / (big_ms * 1e-3) / 1e9,
                                        "peak": load_peaks()["hbm_gbs"], "unit": "GB/s"}},
           "sequence_batch_us": seq_ms * 1e3}
    if ref is not None:
        sec = ref.ref_time_loader(n, feat, 64, 200)
        row["cpu_baseline"] = {"value": sec / 200 * 1e6, "unit": "us", "cores": cores, "kind": "reference",
                               "sample": "200 get_batch calls of the same loader shape (host stacking)"}
    out["dataloader"] = row

    # -- checkpoint of a 4096 x 4096 Linear with its AdamW state ----------------------------------------
    from nnb.checkpoint import load_checkpoint, save_checkpoint
    from nnb.nn import AdamW, Linear, Sequential
    m = Sequential(Linear(4096, 4096, np.random.default_rng(4), dev))
    opt = AdamW(m.parameters())
    for prm in m.parameters():
        prm.grad.fill_(0.5)
        prm.grad_fresh = False
    opt.step()
    torch.cuda.synchronize()
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "ck.nnck")
        t0 = time.perf_counter()
        save_checkpoint(path, m, opt, step=1)
        load_checkpoint(path, m, opt)
        torch.cuda.synchronize()
        sec = time.perf_counter() - t0
        nbytes = os.path.getsize(path)
        row = {"metric": "checkpoint save+load s", "value": sec, "unit": "s",
               "config": {"workload": "Sequential{Linear(4096, 4096)} + AdamW state (NNCK v1, 201 MB), local temp dir"},
               "mb_per_s": 2 * nbytes / sec / 1e6, "bytes": nbytes}
        if ref is not None:
            rsec = ref.ref_time_checkpoint(os.path.join(tmp, "ref.nnck").encode(), 4096, 4096)
            row["cpu_baseline"] = {"value": rsec, "unit": "s", "cores": cores, "kind": "reference",
                                   "sample": "one save + load of the same model and optimizer"}
    out["checkpoint"] = row

    # -- general conv: dilation 2, groups 4 ---------------------------------------------------------------
    Nc, Cin, Hc, Wc, Cout, kk, stride, pad, dil, groups = 64, 32, 28, 28, 64, 3, 1, 2, 2, 4
    xc = torch.randn(Nc, Cin, Hc, Wc, device=dev, generator=g)
    wc = torch.randn(Cout, Cin // groups, kk, kk, device=dev, generator=g) * 0.1
    bc = torch.randn(Cout, device=dev, generator=g)
    gc = torch.randn(Nc, Cout, Hc, Wc, device=dev, generator=g)

    def conv():
        X, Wt, B = Value.leaf(xc, True), Value.leaf(wc, True), Value.leaf(bc, True)
        Y = F.conv2d(X, Wt, B, stride, pad, dilation=dil, groups=groups)
        Y.backward(gc)

    conv_ms = events(conv, 10)
    flops = 3 * 2 * Nc * Cout * Hc * Wc * (Cin // groups) * kk * kk
    row = {"metric": "conv2d (dilation 2, groups 4) fwd+bwd ms", "value": conv_ms, "unit": "ms",
           "config": {"workload": "x [64, 32, 28, 28], w [64, 8, 3, 3], pad 2, dilation 2, groups 4, eager"},
           "algorithmic_tflops": flops / (conv_ms * 1e-3) / 1e12}
    if ref is not None:
        xa, wa, ba, ga2 = (t.cpu().numpy().ravel() for t in (xc, wc, bc, gc))
        ya, dxa, dwa, dba = (np.zeros(a.size, np.float32) for a in (ga2, xa, wa, ba))
        t0 = time.perf_counter()
        ref.ref_conv2d_ex(Nc, Cin, Hc, Wc, Cout, kk, kk, stride, pad, dil, groups, *(orc.ptr(a) for a in
                                                                                  (xa, wa, ba, ga2, ya, dxa, dwa, dba)))
        row["cpu_baseline"] = {"value": (time.perf_counter() - t0) * 1e3, "unit": "ms", "cores": cores,
                               "kind": "reference", "sample": "one fwd+bwd of the same shape"}
    out["conv_general"] = row
    return out


def cpu_baselines(cores: int | None = None):
    """The reference's own CPU code (oracle/_ref) on the host cores for configs 1, 2, 3 and 5, each a
    bounded sample (a few seconds)."""
    import numpy as np

    from oracle import orc

    ref = orc.ref()
    if ref is None:
        return {"unavailable": "reference library not built"}
    cores = cores or os.cpu_count() or 1
    ref.ref_set_threads(cores)
    out = {"cores": cores, "kind": "reference"}
    P = orc.ptr
    # config 1
    ab = orc.uniform(0, 2 * 512 * 512)
    sec = ref.ref_time_matmul(512, 512, 512, P(ab[:512 * 512]), P(ab[512 * 512:]), 50)
    out["config1_matmul512_tflops"] = 2 * 512 ** 3 / sec / 1e12
    # config 2
    N = 64
    x = orc.uniform(50, N * 784, 0.0, 1.0)
    labels = orc.integers(51, N, 0, 9)
    sizes = [32 * 9, 32, 64 * 288, 64, 128 * 3136, 128, 1280, 10]
    params = np.concatenate([orc.uniform(60 + i, n, -0.05, 0.05) for i, n in enumerate(sizes)])
    loss, logits, grads = np.zeros(1, np.float32), np.zeros((N, 10), np.float32), np.zeros_like(params)
    ts = []
    for _ in range(4):
        t0 = time.perf_counter()
        ref.ref_cnn_fwd_bwd(N, P(x), P(labels), P(params), P(loss), P(logits), P(grads))
        ts.append(time.perf_counter() - t0)
    out["config2_cnn_ms_per_step"] = statistics.median(ts[1:]) * 1e3
    # config 3 (full size)
    Na, T, D, H = 32, 256, 512, 8
    q, k, v, g = (orc.normal(70 + i, Na * T * D) for i in range(4))
    o, dq, dk, dv = (np.zeros(Na * T * D, np.float32) for _ in range(4))
    ts = []
    for _ in range(2):
        t0 = time.perf_counter()
        ref.ref_attention(Na, T, T, D, H, P(q), P(k), P(v), None, 1, P(g), P(o), P(dq), P(dk), P(dv))
        ts.append(time.perf_counter() - t0)
    out["config3_attention_ms_per_step"] = min(ts) * 1e3
    # config 5 on 8 of the 64 sequences (one virtual shard), one training step
    cfg = (4096, 512, 8, 4, 512)
    n_params = 16808960
    prm = orc.uniform(80, n_params, -0.04, 0.04)
    ids = orc.integers(81, 8 * 513, 0, 4095).reshape(8, 513)
    xi, yi = np.ascontiguousarray(ids[:, :512]), np.ascontiguousarray(ids[:, 1:])
    losses, prm_out = np.zeros(1, np.float32), np.zeros_like(prm)
    t0 = time.perf_counter()
    n = ref.ref_transformer_train(*cfg, 8, 512, P(prm), P(xi), P(yi), 3e-4, 1e-2, 1, P(losses), None, P(prm_out))
    sec = time.perf_counter() - t0
    out["config5_transformer_tokens_per_s"] = 8 * 512 / sec if n == n_params else None
    out["sample"] = ("config 1: 50 calls; config 2: 3 steps after 1; config 3: best of 2 full fwd+bwd; config 5: "
                     "one AdamW step on 8 of the 64 sequences (4096 tokens)")
    return out


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "next":
            if rank == 0:
                print(json.dumps(run_next_rows(local_rank, with_cpu=not args.no_cpu_baseline)), flush=True)
        elif args.workload in ("cnn", "attention"):
            if rank == 0:
                fn = run_cnn if args.workload == "cnn" else run_attention
                print(json.dumps(fn(max(args.t_steps, 10), args.t_warmup, local_rank)), flush=True)
        elif args.workload == "transformer":
            t = run_transformer(args.t_steps, args.t_warmup, rank, world, local_rank)
            if rank == 0:
                t.update({"n_gpus": world, "higher_is_better": True, "vs_baseline": None, "dtype": "tf32x3",
                          "data": "synthetic token ids (torch generator, fixed seed)"})
                print(json.dumps(t), flush=True)
        else:
            run_nnb(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
