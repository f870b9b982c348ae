#!/usr/bin/env python3
"""Benchmark of the hot path on B200: config 0 of the baseline, the Q4_K decode GEMV.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the hot path over one activation: the activation quantization
(quantizeAct) and the Q4_K GEMV of a 4096 x 4096 weight (config 0), one kernel (the GEMV
quantizes the f32 activation itself).  Weights rotate over 32
seeded copies (302 MB, larger than the 126 MB L2), so every step streams its weight from HBM.
`value` is the whole-job throughput in GB/s of algorithmic bytes (weight + x + y = 9,469,952 B
per step) with everything resident in HBM; `e2e` is the same metric through the public host-
buffer entry point zllm_matvec (x copied in, y copied out every step).  Under torchrun each rank
runs its own weights (independent matrices: weak scaling, no collective on the data path).

`--impl reference` times the CPU implementation of the same path on the host cores: the
reference is JavaScript and no Node.js runtime exists on these machines, so the timed
implementation is the C restatement of its plain-JS kernels (oracle/, OpenMP over rows).
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

ROWS, COLS = 4096, 4096
NCOPY = 32
SEED = 20261201
W_BYTES = ROWS * COLS // 256 * 144                      # 9,437,184
ALGO_BYTES = W_BYTES + COLS * 4 + ROWS * 4             # + x (f32) + y (f32) = 9,469,952
METRIC = "Q4_K GEMV HBM GB/s"
UNIT = "GB/s"


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_from_profile():
    """dram bytes (read + write) per launch from the committed ncu summary of this kernel, if any."""
    p = os.path.join(ROOT, "profiles", "gemv_q4k_4096x4096.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi sampler running during the timed region (the profiling recipe's query)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        rows = [l.strip().split(", ") for l in self.f.read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(seconds: float, nthreads: int):
    """The oracle's Q4_K matvec (C restatement of ref-kernels.js:196-242), OpenMP over rows."""
    import oracle as O
    try:
        lib = O.lib(O.build(native=True))
        kind_note = "-march=native"
    except Exception:
        lib = O.lib()
        kind_note = "portable"
    from zerollm_b200 import ggml, synth
    rng = np.random.default_rng(SEED)
    w = synth.quant_blocks(ggml.Q4_K, ROWS, COLS, rng, "bench").reshape(-1)
    x = rng.standard_normal(COLS).astype(np.float32)
    O.matvec(ggml.Q4_K, w, ROWS, COLS, x, nthreads=nthreads, library=lib)
    n, t0 = 0, time.perf_counter()
    while True:
        O.matvec(ggml.Q4_K, w, ROWS, COLS, x, nthreads=nthreads, library=lib)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": round(ALGO_BYTES * n / el / 1e9, 3), "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": f"{n} Q4_K {ROWS}x{COLS} matvecs (one weight, cache-warm) in {el:.1f} s; C restatement of the "
                      f"reference's plain-JS kernel ({kind_note}), the reference itself is JavaScript and no Node.js is installed"}


def dist_setup(n_gpus):
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def run_reference(args, world, rank):
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    import oracle as O
    from zerollm_b200 import ggml, synth
    try:
        lib = O.lib(O.build(native=True))
    except Exception:
        lib = O.lib()
    rng = np.random.default_rng(SEED)
    w = synth.quant_blocks(ggml.Q4_K, ROWS, COLS, rng, "bench").reshape(-1)
    x = rng.standard_normal(COLS).astype(np.float32)
    for _ in range(args.warmup):
        O.matvec(ggml.Q4_K, w, ROWS, COLS, x, nthreads=nthreads, library=lib)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.matvec(ggml.Q4_K, w, ROWS, COLS, x, nthreads=nthreads, library=lib)
    el = time.perf_counter() - t0
    v = ALGO_BYTES * args.steps / el / 1e9
    sample = (f"{args.steps} Q4_K {ROWS}x{COLS} matvecs per run, one weight (cache-warm); C restatement of the reference's "
              f"plain-JS kernels (the reference is JavaScript; no Node.js runtime on this box)")
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/f64", "data": "synthetic",
            "config": {"workload": "config0: Q4_K GEMV 4096x4096, batch 1", "rows": ROWS, "cols": COLS, "seed": SEED},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": nthreads, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    import ctypes as C

    import torch

    from zerollm_b200 import ggml, synth
    from zerollm_b200.kernels import Context, Weight
    from zerollm_b200.lib import check

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    ctx = Context(local)
    L = ctx.lib
    rng = np.random.default_rng(SEED + 7919 * rank)
    weights = [Weight(ctx, ggml.Q4_K, ROWS, COLS, synth.quant_blocks(ggml.Q4_K, ROWS, COLS, rng, "bench").reshape(-1))
               for _ in range(NCOPY)]
    x_np = rng.standard_normal(COLS).astype(np.float32)
    x = torch.as_tensor(x_np).to(dev)
    xq = torch.empty(COLS, dtype=torch.int8, device=dev)
    xd = torch.empty(COLS // 32, dtype=torch.float32, device=dev)
    xs = torch.empty(COLS // 32, dtype=torch.int32, device=dev)
    y = torch.empty((NCOPY, ROWS), dtype=torch.float32, device=dev)
    P = lambda t: C.c_void_p(t.data_ptr())
    stream = torch.cuda.Stream(device=dev)

    def enqueue(n, with_quant=True, offset=0):
        """n steps; with_quant: f32 activation in (quantized inside the GEMV), else the pre-quantized one."""
        s = C.c_void_p(stream.cuda_stream)
        for i in range(n):
            j = (i + offset) % NCOPY
            if with_quant:
                check(L.zllm_mm(ctx.h, weights[j].h, None, None, None, P(x), 1, C.c_void_p(y[j].data_ptr()), ROWS,
                                None, s), ctx.h)
            else:
                check(L.zllm_mm(ctx.h, weights[j].h, P(xq), P(xd), P(xs), None, 1, C.c_void_p(y[j].data_ptr()), ROWS,
                                None, s), ctx.h)

    def graph(n, with_quant=True):
        enqueue(2, with_quant)                      # set kernel attributes outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            enqueue(n, with_quant)
        return g

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([v], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return v

    check(L.zllm_quantize_act(ctx.h, P(x), COLS, 1, P(xq), P(xd), P(xs), C.c_void_p(stream.cuda_stream)), ctx.h)
    if args.profile:
        # plain launches (no graph) for an ncu capture: warm-up then `steps` GEMV launches
        enqueue(args.warmup)
        enqueue(args.steps)
        torch.cuda.synchronize()
        ctx.sync()
        if rank == 0:
            print(json.dumps({"profile_run": True, "launches": args.warmup + args.steps}))
        ctx.close()
        return

    g_warm = graph(max(args.warmup, 1))
    g_main = graph(args.steps)
    g_kern = graph(args.steps, with_quant=False)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # ---------------------------------------------------------------- timed region (value)
    with torch.cuda.stream(stream):
        for _ in range(3):
            g_warm.replay()
    barrier()
    clocks = Clocks(local)
    with clocks:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            g_main.replay()
            ev1.record(stream)
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ctx.sync()

    # ---------------------------------------------------------------- the same GEMV on a pre-quantized activation
    with torch.cuda.stream(stream):
        g_kern.replay()
        ev0.record(stream)
        g_kern.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    kern_ms = ev0.elapsed_time(ev1) / args.steps
    ctx.sync()

    # parity spot check of the timed outputs against the oracle (row sample)
    import oracle as O
    ref = O.matvec(ggml.Q4_K, np.ascontiguousarray(synth.quant_blocks(ggml.Q4_K, ROWS, COLS, np.random.default_rng(SEED + 7919 * rank), "bench")).reshape(-1),
                   ROWS, COLS, x_np, nthreads=os.cpu_count() or 1, r1=256)[:256]
    got = y[0, :256].cpu().numpy()
    parity = float(np.abs(got - ref).max() / np.abs(ref).max())

    # ---------------------------------------------------------------- e2e through the host-buffer entry point
    xh = torch.empty(COLS, dtype=torch.float32).pin_memory()
    xh.copy_(torch.as_tensor(x_np))
    yh = torch.empty(ROWS, dtype=torch.float32).pin_memory()
    e_steps = max(20, min(args.steps, 500))
    for i in range(3):
        check(L.zllm_matvec(ctx.h, weights[i].h, P(xh), 1, P(yh)), ctx.h)
    barrier()
    cs = torch.cuda.ExternalStream(ctx.stream, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    for i in range(e_steps):
        check(L.zllm_matvec(ctx.h, weights[i % NCOPY].h, P(xh), 1, P(yh)), ctx.h)
    e1.record(cs)
    e1.synchronize()
    e_ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()

    if rank == 0:
        peak, peak_kind = measured_peaks()
        value = ALGO_BYTES * args.steps * world / (ms / 1e3) / 1e9
        # every launch of the timed region is the one GEMV kernel: its average duration is ms / steps
        achieved = ALGO_BYTES / (ms / args.steps / 1e3) / 1e9
        traffic = traffic_from_profile()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/f64", "data": "synthetic",
            "config": {"workload": "config0: Q4_K GEMV 4096x4096, batch 1 (quantizeAct fused into the matvec kernel)",
                       "rows": ROWS,
                       "cols": COLS, "weight_copies": NCOPY, "seed": SEED, "parallelism": f"replicas{world}",
                       "l2": f"inputs larger than L2: {NCOPY} rotating weight copies ({NCOPY * W_BYTES / 1e6:.0f} MB)",
                       "algorithmic_bytes_per_step": ALGO_BYTES, "graph": "CUDA graph of all timed steps, PDL edges"},
            "e2e": {"value": round(ALGO_BYTES * e_steps * world / (e_ms / 1e3) / 1e9, 2), "unit": UNIT,
                    "h2d_bytes_per_step": COLS * 4, "d2h_bytes_per_step": ROWS * 4,
                    "steps": e_steps, "api": "zllm_matvec (host buffers, pinned)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "kq_gemv_kernel<Q4_K, one token> (in-kernel activation quantization)",
                         "kernel_us": round(ms / args.steps * 1e3, 3),
                         "prequantized_kernel_us": round(kern_ms * 1e3, 3),
                         "algorithmic_bytes_per_launch": ALGO_BYTES},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "parity": {"max_rel_err_vs_oracle": parity, "rows_checked": 256},
        }
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds, os.cpu_count() or 1)
        print(json.dumps(line), flush=True)
    del g_warm, g_main, g_kern
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile", action="store_true", help="plain launches without graphs or timing, for ncu")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
