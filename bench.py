#!/usr/bin/env python3
"""Benchmark of the f32 matmul hot path (Momiru's frozen-plan GEMM node) on B200.

Workload (default): M = N = K = 8192 f32 with the fused epilogue
C = ReLU(A @ B + bias); A, B uniform[-1,1) (SplitMix64 seeds 1, 2), bias
normal(0, 0.1) (seed 3), StrictFp32 math (3xTF32 on tcgen05). One step is one
bound replay of that node. On N GPUs the output columns are dealt out in
256-column tile units; each rank computes its column block and its GEMM
epilogue stores every finished tile into all ranks' replicas of C over NVLink,
so every rank holds the whole C (total work fixed: strong scaling).

  value   TFLOP/s of the whole job, device-timed (inputs resident in HBM)
  e2e     the same metric through the public API with host buffers: per step
          H2D of A, B, bias from pinned memory, the replay, D2H of C
  roofline the dominant kernel's achieved TFLOP/s against the TF32-derived
          peak (measured bf16 dense peak / 2, divided by 3 for 3xTF32)

`--impl reference` times the reference's CPU GEMM (restated, oracle/) on the
host cores on a bounded row sample of the same workload.
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

FLUSH_NOTE = "inputs (A,B: 512 MiB) larger than the 126 MB L2; no flush needed"
METRIC = "f32 GEMM TFLOP/s @8192^3 (C=ReLU(A@B+bias)), % of TF32 peak"


def workload_config(n: int, world: int) -> dict:
    return {"workload": f"gemm_{n}x{n}x{n}_bias_relu", "m": n, "n": n, "k": n,
            "parallelism": f"column-block x{world}" + (" + replicated output (epilogue peer stores)" if world > 1 else ""),
            "l2": FLUSH_NOTE}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--mode", choices=["strict", "tf32"], default="strict")
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--panels", type=int, default=0,
                    help="row panels of the host-buffer e2e path (0 = one per 512 rows, at most 16)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--library-context", action="store_true",
                    help="also time cuBLAS (torch.matmul, TF32 allowed / strict FP32) on the same operands, "
                         "outside the timed region, as a library reference point")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--workload", choices=["c3", "c1", "c2", "c4", "c5a", "c5b"], default="c3",
                    help="c3 (default) is the headline line; the others are the remaining configurations, "
                         "measured the same way and reported one JSON line each")
    ap.add_argument("--gemv-m", type=int, choices=[1, 4, 16], default=0,
                    help="c5b: time only this M (default: M = 1, 4 and 16)")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p.get("hbm_gbs", 6650.0), "bf16_tflops": p.get("bf16_tflops", 1590.0),
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", 1400.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampled every 25 ms while `active` is set (a short timed
    region at several GPUs still gets a few samples)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.active = False
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "25",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            if self.active:
                self.samples.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for i, n in enumerate(names):
                if len(s) > 5 + i and s[5 + i].lower().startswith("active"):
                    reasons.add(n)
        pw = [float(s[3]) for s in self.samples if s[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples),
                "power_w_max": max(pw) if pw else None}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def single_thread_sample(a, b, seconds: float = 4.0) -> dict:
    """The reference's own dispatch: one caller thread (CpuDispatch
    CallerThread / SingleThread, cpu.rs:1372-1374) running gemm_avx2 over a
    row sample of the same GEMM."""
    from oracle import oracle as O
    n, k = b.shape[1], a.shape[1]
    t0 = time.perf_counter()
    O.gemm_avx2_restated(a[:1], b, 0, 1, 1)
    per_row = max(time.perf_counter() - t0, 1e-4)
    rows = max(1, min(a.shape[0], int(seconds / per_row)))
    t0 = time.perf_counter()
    O.gemm_avx2_restated(a[:rows], b, 0, rows, 1)
    dt = time.perf_counter() - t0
    return {"value": 2.0 * rows * n * k / dt / 1e12, "unit": "TFLOP/s", "cores": 1,
            "sample": f"{rows} of {a.shape[0]} output rows, one thread (restated gemm_avx2), {dt:.1f} s"}


def cpu_baseline_sample(a, b, bias, seconds: float):
    """The reference's CPU GEMM (gemm_avx2 loop structure, restated in oracle/)
    on all host threads over a bounded row sample of the same workload, plus
    the single-thread figure of the reference's own dispatch."""
    from oracle import oracle as O
    O.build()
    n = a.shape[1]
    nthreads = os.cpu_count() or 1
    rows = nthreads
    t0 = time.perf_counter()
    O.gemm_avx2_restated(a[:rows], b, 0, rows, nthreads)
    dt = time.perf_counter() - t0
    per_row_batch = max(dt, 1e-3)
    reps = max(1, int(seconds / per_row_batch))
    rows_total = min(a.shape[0], rows * reps)
    t0 = time.perf_counter()
    O.gemm_avx2_restated(a[:rows_total], b, 0, rows_total, nthreads)
    dt = time.perf_counter() - t0
    flops = 2.0 * rows_total * n * a.shape[1]
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": nthreads, "kind": "port",
            "sample": f"{rows_total} of {a.shape[0]} output rows of the {a.shape[0]}x{n}x{a.shape[1]} GEMM "
                      f"(restated gemm_avx2, -O3 -mavx2 -ffp-contract=off, row-sharded), {dt:.1f} s",
            "cpu_model": cpu_model(), "single_thread": single_thread_sample(a, b)}


def library_context(fn_by_mode: dict, flops: float, iters: int) -> dict:
    """cuBLAS on the same operands (torch.matmul), timed with CUDA events after
    two warm-ups over as many back-to-back calls as the measured region had
    steps (a long run settles at the power cap, a short burst does not): a
    reference point from the vendor library, not this path."""
    import torch
    out = {}
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        for label, (allow_tf32, fn) in fn_by_mode.items():
            torch.backends.cuda.matmul.allow_tf32 = allow_tf32
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            out[label] = flops / (e0.elapsed_time(e1) / iters * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    out["unit"] = "TFLOP/s"
    out["iters"] = iters
    out["what"] = "cuBLAS through torch.matmul on the same device tensors (context only)"
    return out


def dist_init(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # NCCL here only carries the handshakes, the max-over-ranks timings and
    # the input all-gather of the e2e leg: no NVLink multicast (NVLS) buffers,
    # which would stay bound to every rank's memory for the whole run.
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    return rank, world, local


def run_reference(args, rank, world):
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    from momiru_b200 import rng
    from oracle import oracle as O
    O.build()
    n = args.size
    nthreads = os.cpu_count() or 1
    a = rng.randu((n, n), 1)
    b = rng.randu((n, n), 2)
    bias = rng.randn((n,), 3, 0.1)

    def step(rows):
        # the reference's three nodes: MatMul (gemm_avx2), Add(bias), Relu
        c = O.gemm_avx2_restated(a[:rows], b, 0, rows, nthreads)
        return O.relu(c + bias)

    # size the per-step row sample so the whole run takes a few minutes at most
    t0 = time.perf_counter()
    step(nthreads)
    dt = max(time.perf_counter() - t0, 1e-3)
    total_steps = args.steps + args.warmup
    budget = 120.0 / max(total_steps, 1)
    rows = min(n, max(nthreads, int(nthreads * budget / dt)))
    for _ in range(args.warmup):
        step(rows)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step(rows)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    single_thread = single_thread_sample(a, b)
    flops = 2.0 * rows * n * n
    value = flops / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value,
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (SplitMix64 uniform[-1,1) A,B; normal(0,0.1) bias)",
        "config": workload_config(n, world),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": nthreads, "kind": "port",
                         "sample": f"{rows} of {n} output rows per step (restated gemm_avx2 + bias + ReLU, "
                                   f"row-sharded over {nthreads} threads)",
                         "cpu_model": cpu_model(), "single_thread": single_thread},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_workload(args, rank, world, local):
    """The non-headline configurations, device-timed with CUDA events.

    c1  512^3 row-major                        (TFLOP/s, tensor roofline)
    c2  [64,256,256] @ [256,256] broadcast     (TFLOP/s)
    c4  A = X^T view, B = W[:, :11008] view    (TFLOP/s)
    c5a [512,1024,1024] @ [512,1024,1024]      (TFLOP/s; batch-sharded over ranks, no collective)
    c5b [M,4096] @ [4096,4096], M in 1,4,16    (HBM GB/s; four B copies rotate so L2 cannot serve them)
    """
    import torch
    import torch.distributed as dist
    from momiru_b200 import (AccuracyContract, BoundGemm, DeviceBuffer, DeviceView, Epilogue, KernelMathMode,
                             MatMulNode, rng)
    from momiru_b200.sharding import batch_shards
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    dev = local
    mode = KernelMathMode.StrictFp32 if args.mode == "strict" else KernelMathMode.Tf32
    acc = AccuracyContract.StrictFp32 if args.mode == "strict" else AccuracyContract.AllowTf32
    node = MatMulNode(math_mode=mode, accuracy=acc)
    stream = torch.cuda.current_stream()
    peaks = load_peaks()
    lines = []

    def dv(arr):
        return DeviceView.from_host(arr, dev)

    def timed(handles, flops, bytes_, name, cfg, bound, lib=None):
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        for _ in range(max(args.warmup, 3)):
            for h in handles:
                h.replay()
        w1.record(stream)
        torch.cuda.synchronize()
        # a step of a few microseconds: time enough of them that the clock
        # sampler (25 ms period) sees the timed region
        est_ms = w0.elapsed_time(w1) / (max(args.warmup, 3) * len(handles))
        steps = max(args.steps, int(0.6 / max(est_ms * 1e-3, 1e-7)) + 1)
        if world > 1:
            t = torch.tensor([steps], device=f"cuda:{dev}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            steps = int(t.item())
        clocks = ClockSampler(dev)
        clocks.start()
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.active = True
        e0.record(stream)
        for i in range(steps):
            handles[i % len(handles)].replay()
        e1.record(stream)
        torch.cuda.synchronize()
        clocks.active = False
        clocks.stop()
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=f"cuda:{dev}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        for h in handles:
            h.quiesce_or_abort(60)
        tf32_peak = peaks["bf16_tflops"] / 2.0
        if bound == "hbm":
            value, unit, peak = bytes_ / (ms * 1e-3) / 1e9, "GB/s", peaks["hbm_gbs"]
        else:
            value, unit = flops / (ms * 1e-3) / 1e12, "TFLOP/s"
            peak = tf32_peak / 3.0 if args.mode == "strict" else tf32_peak
        per_rank = value / world
        lines.append({
            "metric": name, "value": value, "unit": unit, "n_gpus": world, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
            "scaling": ("weak" if args.workload == "c5a" else "strong" if args.workload == "c4" else "replicas")
                       if world > 1 else "n/a",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (SplitMix64)", "config": cfg,
            "math": "3xTF32 (StrictFp32)" if args.mode == "strict" else "TF32",
            "family": handles[0].family,
            "roofline": {"bound": bound, "achieved": per_rank, "peak": peak, "unit": unit, "frac": per_rank / peak,
                         "peak_basis": "measured HBM copy" if bound == "hbm" else
                         f"measured bf16 dense / 2{' / 3' if args.mode == 'strict' else ''}"},
            "clocks": clocks.summary(),
        })
        if lib is not None and args.library_context:
            lines[-1]["library_context"] = library_context(lib, flops / world, steps)

    w = args.workload
    if w == "c1":
        a, b = dv(rng.randu((512, 512), 1)), dv(rng.randu((512, 512), 2))
        out = DeviceView.empty((512, 512), dev)
        timed([BoundGemm(node, a, b, out, stream=stream.cuda_stream)], 2.0 * 512 ** 3, 3 * 4 * 512 ** 2,
              "C1 512^3 f32 GEMM TFLOP/s", {"workload": "c1_512^3", "l2": "resident (small case)"}, "tensor")
    elif w == "c2":
        a, b = dv(rng.randn((64, 256, 256), 1)), dv(rng.randn((256, 256), 2))
        out = DeviceView.empty((64, 256, 256), dev)
        timed([BoundGemm(node, a, b, out, stream=stream.cuda_stream)], 2.0 * 64 * 256 ** 3,
              4 * (2 * 64 * 256 * 256 + 256 * 256), "C2 batched 64x256^3 (B broadcast) TFLOP/s",
              {"workload": "c2_batch64_256^3_bcast", "l2": "resident (33.8 MB)"}, "tensor")
    elif w == "c4":
        x, wt = dv(rng.randn((4096, 4096), 1, 0.02)), dv(rng.randn((4096, 12288), 2, 0.02))
        out = DeviceView.empty((4096, 11008), dev)
        xt, wtt, ot = x.torch_view(), wt.torch_view(), out.torch_view()
        lhs, rhs = x.transpose(), wt.narrow(1, 0, 11008)
        cfg = {"workload": "c4_xT_4096_wslice_11008", "l2": "inputs 245 MB > L2"}
        if world > 1:
            # Column blocks of 256-column units, each rank keeping its block of
            # the output (no replication, so no collective): strong scaling.
            from momiru_b200.sharding import column_block_views
            rhs, out_l, _, c0, c1 = column_block_views(node, lhs, rhs, out, None, rank, world)
            cfg["parallelism"] = f"column-block x{world}, output kept sharded, no collective"
            cfg["columns"] = [c0, c1]
            g = BoundGemm(node, lhs, rhs, out_l, stream=stream.cuda_stream)
        else:
            g = BoundGemm(node, lhs, rhs, out, stream=stream.cuda_stream)
        lib = {"cublas_tf32": (True, lambda: torch.matmul(xt.t(), wtt[:, :11008], out=ot)),
               "cublas_fp32": (False, lambda: torch.matmul(xt.t(), wtt[:, :11008], out=ot))}
        timed([g], 2.0 * 4096 * 4096 * 11008, 4 * (4096 * 4096 + 2 * 4096 * 11008),
              "C4 strided views 4096x4096x11008 TFLOP/s", cfg, "tensor", lib)
        if world > 1:
            # every block against the oracle on sampled rows: gather the blocks
            # on rank 0 (after the timed region)
            blk = out.torch_view()[:, c0:c1].contiguous()
            sizes = [torch.tensor([blk.shape[1]], device=f"cuda:{dev}") for _ in range(world)]
            dist.all_gather(sizes, torch.tensor([blk.shape[1]], device=f"cuda:{dev}"))
            widest = max(int(t.item()) for t in sizes)
            pad = torch.zeros((4096, widest), dtype=torch.float32, device=f"cuda:{dev}")
            pad[:, :blk.shape[1]] = blk
            blocks = [torch.empty_like(pad) for _ in range(world)]
            dist.all_gather(blocks, pad)
            if rank == 0:
                full = torch.cat([b[:, :int(t.item())] for b, t in zip(blocks, sizes)], dim=1).cpu().numpy()
                lines[-1]["parity"] = c4_sampled_parity(full, x.to_host(), wt.to_host()[:, :11008], args.mode)
    elif w == "c5a":
        b0, b1 = batch_shards(512, world)[rank]
        nb = b1 - b0
        a = DeviceView.empty((nb, 1024, 1024), dev)
        b = DeviceView.empty((nb, 1024, 1024), dev)
        # one seeded block of 16 batch entries, repeated over the rank's slice
        # (the values do not change the throughput)
        blk_a = torch.from_numpy(rng.randu((16, 1024, 1024), 1)).to(f"cuda:{dev}")
        blk_b = torch.from_numpy(rng.randu((16, 1024, 1024), 2)).to(f"cuda:{dev}")
        at, bt = a.torch_view(), b.torch_view()
        for i in range(0, nb, 16):
            j = min(16, nb - i)
            at[i:i + j].copy_(blk_a[:j])
            bt[i:i + j].copy_(blk_b[:j])
        out = DeviceView.empty((nb, 1024, 1024), dev)
        ot = out.torch_view()
        lib = {"cublas_tf32": (True, lambda: torch.matmul(at, bt, out=ot)),
               "cublas_fp32": (False, lambda: torch.matmul(at, bt, out=ot))}
        timed([BoundGemm(node, a, b, out, stream=stream.cuda_stream)], 2.0 * 512 * 1024 ** 3,
              4 * 3 * 512 * 1024 ** 2, "C5a batched 512x1024^3 TFLOP/s",
              {"workload": "c5a_batch512_1024^3", "parallelism": f"batch-shard x{world}, no collective",
               "l2": "inputs 4 GiB > L2"}, "tensor", lib)
    elif w == "c5b":
        bs = [dv(rng.randn((4096, 4096), 10 + i)) for i in range(4)]
        for m in ((args.gemv_m,) if args.gemv_m else (1, 4, 16)):
            a = dv(rng.randn((m, 4096), 1))
            outs = [DeviceView.empty((m, 4096), dev) for _ in range(4)]
            hs = [BoundGemm(node, a, bs[i], outs[i], stream=stream.cuda_stream) for i in range(4)]
            timed(hs, 2.0 * m * 4096 * 4096, 4 * (m * 4096 + 4096 * 4096 + m * 4096),
                  f"C5b GEMV M={m} N=K=4096 HBM GB/s",
                  {"workload": f"c5b_gemv_m{m}", "l2": "four 64 MiB B copies rotate (256 MiB > L2)"}, "hbm")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        for line in lines:
            print(json.dumps(line), flush=True)


def replica_digest(t):
    """Order-independent digest of an f32 device tensor's bits: the wrapping
    int64 sums of the words and of the words weighted by position."""
    import torch
    u = t.reshape(-1).view(torch.int32).to(torch.int64)
    w = torch.arange(u.numel(), device=t.device, dtype=torch.int64) % 65521 + 1
    return torch.stack([u.sum(), (u * w).sum()])


def sampled_parity(out_t, a_h, b_h, bias_h, mode, nrows=32):
    """Relative Frobenius error of `nrows` output rows (spread over the whole
    matrix, first and last included) against the oracle."""
    from oracle import oracle as O
    O.build()
    m = a_h.shape[0]
    rows = np.unique(np.linspace(0, m - 1, nrows).astype(np.int64))
    ref = O.matmul(a_h, b_h, bias=bias_h, epilogue=O.EPI_BIAS_RELU, rows=rows, nthreads=os.cpu_count() or 1)
    got = out_t[rows.tolist()].cpu().numpy().astype(np.float64)
    den = float(np.linalg.norm(ref.astype(np.float64)))
    err = float(np.linalg.norm(got - ref) / (den if den > 0 else 1.0))
    tol = 1e-5 if mode == "strict" else 2e-3
    return {"rows": int(len(rows)), "rel_frob": err, "tol": tol, "ok": err <= tol,
            "against": "oracle (restated reference gemm + bias + ReLU)"}


def c4_sampled_parity(full, x_h, w_h, mode, nrows=32):
    """The column-sharded C4 output, gathered from every rank (`full`, host
    [4096, 11008]): `nrows` rows against the oracle on A = X^T, B = W[:, :11008]."""
    from oracle import oracle as O
    O.build()
    rows = np.unique(np.linspace(0, full.shape[0] - 1, nrows).astype(np.int64))
    ref = O.matmul(x_h.T, w_h, rows=rows, nthreads=os.cpu_count() or 1).astype(np.float64)
    got = full[rows].astype(np.float64)
    den = float(np.linalg.norm(ref))
    err = float(np.linalg.norm(got - ref) / (den if den > 0 else 1.0))
    tol = 1e-5 if mode == "strict" else 2e-3
    return {"rows": int(len(rows)), "rel_frob": err, "tol": tol, "ok": err <= tol,
            "against": "oracle (restated reference gemm), blocks of every rank"}


def hg_panels(m, panels):
    """Row-panel boundaries mmr_gemm_bind_host uses: whole 256-row units dealt
    as evenly as possible; by default one panel per two units, at most 16."""
    units = (m + 255) // 256
    np_ = max(1, min(panels or min(16, max(1, units // 2)), max(units, 1)))
    rows = [min(m, (i * (units // np_) + min(i, units % np_)) * 256) for i in range(np_ + 1)]
    return list(zip(rows[:-1], rows[1:]))


def main():
    args = parse()
    rank, world, local = dist_init(args)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload != "c3":
        run_workload(args, rank, world, local)
        return
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    from momiru_b200 import (AccuracyContract, BoundGemm, DeviceBuffer, DeviceView, Epilogue, KernelMathMode,
                             MatMulNode, rng, shard_columns)

    n = args.size
    mode = KernelMathMode.StrictFp32 if args.mode == "strict" else KernelMathMode.Tf32
    node = MatMulNode(math_mode=mode, epilogue=Epilogue.BIAS_RELU,
                      accuracy=AccuracyContract.StrictFp32 if args.mode == "strict" else AccuracyContract.AllowTf32)
    a_h = rng.randu((n, n), 1)
    b_h = rng.randu((n, n), 2)
    bias_h = rng.randn((n,), 3, 0.1)
    dev = torch.device(f"cuda:{local}")
    stream = torch.cuda.current_stream()
    a_t = torch.from_numpy(a_h).to(dev)
    b_t = torch.from_numpy(b_h).to(dev)
    bias_t = torch.from_numpy(bias_h).to(dev)
    c0, c1 = shard_columns(n, world, rank, 256)
    ncols = c1 - c0
    A = DeviceView.contiguous(DeviceBuffer.from_torch(a_t), (n, n))
    if world > 1:
        # Column-block shard per rank; the GEMM epilogue stores every finished
        # tile into all ranks' replicas of C over NVLink (no collective).
        from momiru_b200.sharding import ReplicatedColumnGemm
        out_t = torch.empty((n, n), dtype=torch.float32, device=dev)
        B = DeviceView.contiguous(DeviceBuffer.from_torch(b_t), (n, n))
        BIAS = DeviceView.contiguous(DeviceBuffer.from_torch(bias_t), (n,))
        C = DeviceView.contiguous(DeviceBuffer.from_torch(out_t), (n, n))
        g = ReplicatedColumnGemm(node, A, B, C, BIAS, stream=stream.cuda_stream)
    else:
        out_t = torch.empty((n, n), dtype=torch.float32, device=dev)
        B = DeviceView.contiguous(DeviceBuffer.from_torch(b_t), (n, n))
        BIAS = DeviceView.contiguous(DeviceBuffer.from_torch(bias_t), (n,))
        C = DeviceView.contiguous(DeviceBuffer.from_torch(out_t), (n, n))
        g = BoundGemm(node, A, B, C, BIAS, stream=stream.cuda_stream)

    def step():
        g.replay()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    g.quiesce_or_abort(60)

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.active = True
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        g.replay()
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    clocks.active = False
    if world > 1:
        dist.barrier()
    g.quiesce_or_abort(60)
    total_ms = t_start.elapsed_time(t_end)
    kernel_ms = [s.elapsed_time(e) for s, e in ev]
    ms_step = total_ms / args.steps
    if world > 1:
        tm = torch.tensor([ms_step], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms_step = float(tm.item())
    flops_total = 2.0 * n * n * n
    value = flops_total / (ms_step * 1e-3) / 1e12

    # ---------------------------------------------------------------- e2e
    # Public API with host buffers: this step's inputs copied in from pinned
    # host memory, the result copied back, all inside the timed region. On one
    # GPU that is the host-buffer entry (mmr_gemm_bind_host: rhs and bias in,
    # then lhs by row panels overlapped with the panels' GEMMs and the copies
    # out). Across ranks every byte of the inputs and of the result crosses
    # PCIe once, spread over the ranks' links: each rank copies in its row slab
    # of A (the slabs are then all-gathered over NVLink, since every rank's
    # GEMM reads all of A) and its column block of B and bias, and copies out
    # its column block of the replicated result; the ranks' host blocks
    # together hold C. h2d/d2h bytes are whole-job totals.
    a_pin = torch.from_numpy(a_h).pin_memory()
    b_pin = torch.from_numpy(b_h).pin_memory()
    bias_pin = torch.from_numpy(bias_h).pin_memory()
    c_pin = torch.empty(tuple(out_t.shape), dtype=torch.float32).pin_memory() if world == 1 else None
    h2d = (a_pin.numel() + b_pin.numel() + bias_pin.numel()) * 4
    d2h = out_t.numel() * 4
    e2e_path = "torch copies + replicated GEMM"
    if world == 1:
        from momiru_b200 import HostGemm
        hg = HostGemm(node, a_pin.numpy(), b_pin.numpy(), c_pin.numpy(), bias_pin.numpy(), panels=args.panels,
                      device_ordinal=local, stream=stream.cuda_stream)
        e2e_path = f"mmr_gemm_bind_host, {len(hg_panels(n, args.panels))} row panels, pinned host buffers"

        def e2e_step():
            hg.replay()
    else:
        from cuda.bindings import runtime as cudart
        from momiru_b200.sharding import ReplicatedColumnGemm
        r0, r1 = rank * n // world, (rank + 1) * n // world
        even = n % world == 0  # equal slabs for the all-gather; otherwise every rank copies all of A
        e2e_path = ("each rank: its A row slab in, A all-gathered over NVLink, its B/bias column block in, "
                    "replicated GEMM, its C column block out; two buffer lanes, so step i+1's copies in and "
                    "all-gather run beside step i's GEMM and copy out")

        def copy2d(dst, dpitch, src, spitch, width, rows, kind, st):
            if width and rows:
                err, = cudart.cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, kind, st.cuda_stream)
                if err != cudart.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"cudaMemcpy2DAsync: {err}")

        def make_lane(a_, b_, bias_, out_, g_):
            ev = lambda: torch.cuda.Event()  # noqa: E731
            return {"a": a_, "b": b_, "bias": bias_, "out": out_, "g": g_,
                    "slab": torch.empty((r1 - r0, n), dtype=torch.float32, device=dev),
                    "c": torch.empty((n, ncols), dtype=torch.float32).pin_memory(),
                    "slab_ev": ev(), "in": ev(), "ag": ev(), "gemm": ev(), "out_ev": ev(), "used": False}

        # Lane 1: a second set of device buffers and a second replicated handle
        # (its own replicas, signal array and IPC exchange).
        a2, b2, bias2, out2 = (torch.empty_like(t) for t in (a_t, b_t, bias_t, out_t))
        g2 = ReplicatedColumnGemm(node, DeviceView.contiguous(DeviceBuffer.from_torch(a2), (n, n)),
                                  DeviceView.contiguous(DeviceBuffer.from_torch(b2), (n, n)),
                                  DeviceView.contiguous(DeviceBuffer.from_torch(out2), (n, n)),
                                  DeviceView.contiguous(DeviceBuffer.from_torch(bias2), (n,)),
                                  stream=stream.cuda_stream)
        lanes = [make_lane(a_t, b_t, bias_t, out_t, g), make_lane(a2, b2, bias2, out2, g2)]
        s_in, s_ag, s_out = (torch.cuda.Stream(dev) for _ in range(3))
        fence = torch.zeros(1, dtype=torch.float32, device=dev)
        step_no = [0]

        def e2e_begin():
            # the side streams start after whatever the caller's stream holds
            ev = torch.cuda.Event()
            ev.record(stream)
            for st in (s_in, s_ag, s_out):
                st.wait_event(ev)

        def e2e_end():
            for ln in lanes:
                if ln["used"]:
                    stream.wait_event(ln["out_ev"])

        def e2e_step():
            ln = lanes[step_no[0] % 2]
            step_no[0] += 1
            # copies in, once this lane's previous GEMM has read its inputs
            if ln["used"]:
                s_in.wait_event(ln["gemm"])
            with torch.cuda.stream(s_in):
                if even:
                    ln["slab"].copy_(a_pin[r0:r1], non_blocking=True)
                    ln["slab_ev"].record(s_in)
                else:
                    ln["a"].copy_(a_pin, non_blocking=True)
                copy2d(ln["b"].data_ptr() + 4 * c0, 4 * n, b_pin.data_ptr() + 4 * c0, 4 * n, 4 * ncols, n,
                       cudart.cudaMemcpyKind.cudaMemcpyHostToDevice, s_in)
                if ncols:
                    ln["bias"][c0:c1].copy_(bias_pin[c0:c1], non_blocking=True)
                ln["in"].record(s_in)
            if even:
                with torch.cuda.stream(s_ag):
                    s_ag.wait_event(ln["slab_ev"])
                    dist.all_gather_into_tensor(ln["a"], ln["slab"], async_op=True).wait()
                    ln["ag"].record(s_ag)
            # The GEMM stores into every rank's replica of this lane, so every
            # rank must have finished copying out this lane's previous result:
            # a one-float all-reduce after this rank's own copy out orders it.
            stream.wait_event(ln["in"])
            if even:
                stream.wait_event(ln["ag"])
            if ln["used"]:
                stream.wait_event(ln["out_ev"])
                dist.all_reduce(fence)
            ln["g"].replay()
            ln["gemm"].record(stream)
            s_out.wait_event(ln["gemm"])
            copy2d(ln["c"].data_ptr(), 4 * ncols, ln["out"].data_ptr() + 4 * c0, 4 * n, 4 * ncols, n,
                   cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost, s_out)
            ln["out_ev"].record(s_out)
            ln["used"] = True

    if world == 1:
        def e2e_begin():
            pass

        def e2e_end():
            pass
    e2e_begin()
    for _ in range(1 if world == 1 else 2):  # warm-up (each lane once across ranks)
        e2e_step()
    e2e_end()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks.active = True
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_begin()
    for _ in range(args.e2e_steps):
        e2e_step()
    e2e_end()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks.active = False
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        tm = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        e2e_ms = float(tm.item())
    g.quiesce_or_abort(60)
    if world == 1:
        hg.quiesce_or_abort(60)
        hg.close()
    else:
        g2.quiesce_or_abort(60)
    clocks.stop()

    # ------------------------------------------------------ correctness
    # After the timed regions (which leave the same result in place): every
    # rank's replica must be identical, and rank 0 checks sampled output rows
    # against the oracle (the restated reference CPU GEMM + bias + ReLU).
    digest = replica_digest(out_t)
    replicas_equal = None
    if world > 1:
        everyone = [torch.empty_like(digest) for _ in range(world)]
        dist.all_gather(everyone, digest)
        replicas_equal = all(bool(torch.equal(d, everyone[0])) for d in everyone)
    # the host copy of the result is this rank's column block of the replica
    e2e_host_ok = None
    if world > 1:
        # each lane's host block equals its replica's block, and both lanes
        # computed the same product
        ok = torch.equal(out2, out_t) and all(
            torch.equal(ln["c"], ln["out"][:, c0:c1].cpu()) for ln in lanes if ln["used"])
        bad = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.SUM)
        e2e_host_ok = int(bad.item()) == 0
    parity = None
    if rank == 0:
        parity = sampled_parity(out_t, a_h, b_h, bias_h, args.mode)

    # ----------------------------------------------------------- roofline
    peaks = load_peaks()
    tf32_peak = peaks["bf16_tflops"] / 2.0
    kern_ms = statistics.mean(kernel_ms)
    # the dominant kernel is this rank's GEMM; at N > 1 the replay also holds
    # the fix-up check and the completion handshake, so this is conservative
    shard_flops = 2.0 * n * ncols * n
    achieved = shard_flops / (kern_ms * 1e-3) / 1e12
    peak = tf32_peak / 3.0 if args.mode == "strict" else tf32_peak
    traffic = None
    prof = os.path.join(ROOT, "profiles", "tc_gemm_8192_strict_traffic.json")
    if os.path.exists(prof) and args.size == 8192:
        with open(prof) as f:
            traffic = json.load(f).get(f"{args.mode}_bytes_per_launch_n{world}")

    line = {
        "metric": METRIC, "value": value,
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "math": "3xTF32 (StrictFp32)" if args.mode == "strict" else "TF32",
        "data": "synthetic (SplitMix64 uniform[-1,1) A,B; normal(0,0.1) bias)",
        "config": workload_config(n, world),
        # per step: the GEMM kernel, (3xTF32) the non-finite fix-up check,
        # (N > 1) the replica completion handshake
        "gpu_launches": args.steps * ((2 if args.mode == "strict" else 1) + (1 if world > 1 else 0)),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_basis": (f"{peaks['source']} bf16 dense {peaks['bf16_tflops']} / 2 (TF32 rate)"
                                    + (" / 3 (3xTF32)" if args.mode == "strict" else "")),
                     "kernel_ms": kern_ms, "frac_of_tf32_peak": achieved / tf32_peak},
        "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "path": e2e_path},
        "clocks": clocks.summary(),
        "parity": parity,
        "replicas_equal": replicas_equal,
        "e2e_host_result_equal": e2e_host_ok,
    }
    if args.library_context and world == 1:
        cb = torch.empty_like(out_t)
        line["library_context"] = library_context(
            {"cublas_tf32": (True, lambda: torch.matmul(a_t, b_t, out=cb)),
             "cublas_fp32": (False, lambda: torch.matmul(a_t, b_t, out=cb))}, flops_total, args.steps)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(a_h, b_h, bias_h, args.cpu_seconds)
    g.close()
    if world > 1:
        g2.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
