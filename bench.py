#!/usr/bin/env python3
"""Benchmark of the verified INT8 W8A8 path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints one JSON line (rank 0).  Workloads:

* ``gemm-sweep``: the standalone INT8 GEMM sweep (seeded): A f32 ~ N(0,1)
  quantised per row on the device, B int8 uniform in [-127, 127] with
  per-column scales uniform in [1e-3, 1e-2], M in {1,16,128,512} x (K,N) in
  {(576,1536), (1536,576), (2048,5632), (4096,14336)}; int32 accumulate and
  the requant-LUT int8 output.  One step = the 16 shapes once.  Weights are
  resident in HBM with enough copies per shape that every launch reads them
  cold (each shape's copies total more than 3x the 126 MB L2).

Timing: W untimed warm-up steps, then K steps between barrier +
synchronize, measured with CUDA events on the launching stream, max over
ranks.  ``--impl reference`` times the reference's CPU algorithm (the C
restatement in oracle/, all host cores) on a bounded sample of the same
workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "INT8 decode tok/s + chunked-prefill tok/s at 1/2/4/8 B200; GEMM % roofline"
SWEEP_M = [1, 16, 128, 512]
SWEEP_KN = [(576, 1536), (1536, 576), (2048, 5632), (4096, 14336)]
L2_BYTES = 126 * 1024 * 1024


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm_gbs=d["hbm_gbs"], bf16_tflops=d["bf16_tflops"],
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained"), src="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, src="fallback")


# ---- clocks during the timed region ----------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        """Start sampling and wait (up to 10 s) for the first sample, so the
        timed region that follows is covered."""
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 10 and os.path.getsize(self.path) == 0:
            time.sleep(0.05)
        self.t_start = time.time()

    def mark_end(self):
        """Keep sampling until at least 0.3 s passed since the timed region began."""
        if self.proc is not None:
            while time.time() - self.t_start < 0.3:
                time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return dict(sm_mhz=statistics.median(r[0] for r in rows), sm_max_mhz=max(r[1] for r in rows),
                    reasons=reasons, samples=len(rows))


# ---- distributed plumbing -----------------------------------------------------------
def dist_init():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, local, world


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- the GEMM sweep -------------------------------------------------------------------
def sweep_shapes():
    return [(m, k, n) for (k, n) in SWEEP_KN for m in SWEEP_M]


def gemm_bytes(m, k, n, out_bytes):
    return m * k + k * n + 4 * m + 4 * n + out_bytes * m * n


class SweepData:
    """Device buffers of the sweep: A f32, its int8 rows + scales, weight copies."""

    def __init__(self, torch, seed=2026):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.items = []
        for (m, k, n) in sweep_shapes():
            ld = (k + 15) // 16 * 16
            A = torch.randn(m, k, generator=g, device="cuda", dtype=torch.float32)
            copies = max(3, math.ceil(3 * L2_BYTES / (n * ld)))
            W = torch.randint(-127, 128, (copies, n, ld), generator=g, device="cuda", dtype=torch.int8)
            if ld != k:
                W[:, :, k:] = 0
            cs = torch.rand(copies, n, generator=g, device="cuda") * 9e-3 + 1e-3
            self.items.append(dict(m=m, k=k, n=n, ld=ld, A=A, W=W, cs=cs, copies=copies,
                                   xq=torch.zeros(m, ld, dtype=torch.int8, device="cuda"),
                                   rs=torch.empty(m, device="cuda"),
                                   out=torch.empty(m * n, dtype=torch.int8, device="cuda")))


def run_sweep_step(comp, data, step, events=None, dom=None):
    """One step: every shape quantises its A rows and runs the GEMM (requant out)."""
    launches = 0
    for i, it in enumerate(data.items):
        c = step % it["copies"]
        comp.quantize_rows_dev(it["A"], it["m"], it["k"], it["xq"], it["ld"], it["rs"])
        if events is not None and i == dom:
            events[0].record()
        comp.bgemm_dev(it["xq"], it["ld"], it["W"][c], it["ld"], it["rs"], it["cs"][c], it["m"], it["k"], it["n"], 1,
                       4, it["out"])
        if events is not None and i == dom:
            events[1].record()
            events[2].append((events[0], events[1]))
            events[0], events[1] = type(events[0])(enable_timing=True), type(events[1])(enable_timing=True)
        launches += 2
    return launches


def bench_gemm_sweep(args, rank, world, peaks):
    import torch
    import __graft_entry__ as G
    P = G.package()
    comp = P.init_compute(0 if world == 1 else int(os.environ.get("LOCAL_RANK", "0")),
                          stream=torch.cuda.current_stream())
    data = SweepData(torch)
    shapes = sweep_shapes()
    # pick the dominant GEMM: time each shape's launch during a warm-up pass
    per = []
    for i, it in enumerate(data.items):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        comp.quantize_rows_dev(it["A"], it["m"], it["k"], it["xq"], it["ld"], it["rs"])
        e0.record()
        comp.bgemm_dev(it["xq"], it["ld"], it["W"][0], it["ld"], it["rs"], it["cs"][0], it["m"], it["k"], it["n"], 1,
                       4, it["out"])
        e1.record()
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1))
    dom = max(range(len(per)), key=lambda i: per[i])
    for s in range(args.warmup):
        run_sweep_step(comp, data, s)
    comp.sync()
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    evs = [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True), []]
    launches = 0
    t0.record()
    for s in range(args.steps):
        launches += run_sweep_step(comp, data, args.warmup + s, evs, dom)
    t1.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    barrier(world)
    clk = clocks.stop()
    comp.sync()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, world)
    ops_step = sum(2.0 * m * k * n for (m, k, n) in shapes)
    value = ops_step * world / (ms / 1e3) / 1e12
    m, k, n = shapes[dom]
    dom_ms = statistics.mean(a.elapsed_time(b) for a, b in evs[2])
    ops = 2.0 * m * k * n
    byts = gemm_bytes(m, k, n, 1)
    i8_peak = 2.0 * peaks["bf16_tflops"]
    ridge = i8_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if ops / byts > ridge:
        roof = dict(bound="tensor", achieved=ops / (dom_ms / 1e3) / 1e12, peak=i8_peak, unit="TOPS")
        peak_note = f"2 x {peaks['src']} bf16 dense TFLOP/s (int8 dense rate = 2 x bf16)"
    else:
        roof = dict(bound="hbm", achieved=byts / (dom_ms / 1e3) / 1e9, peak=peaks["hbm_gbs"], unit="GB/s")
        peak_note = f"{peaks['src']} HBM copy bandwidth"
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = traffic_for(f"gemm_{m}x{k}x{n}")
    roof["kernel"] = f"{'tcgen05' if comp.tc_enabled and m > 8 else ('gemv' if m <= 8 else 'simt')} GEMM {m}x{k}x{n}"
    roof["peak_source"] = peak_note
    roof["algorithmic_per_launch"] = dict(ops=ops, bytes=byts)
    line = dict(metric=METRIC, value=value, unit="TOPS (int8 ops/s, GEMM sweep)", n_gpus=world, steps=args.steps,
                warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling="weak", vs_baseline=None,
                dtype="int8 x int8 -> int32", data="synthetic (seeded)",
                config=dict(workload="gemm-sweep: M{1,16,128,512} x (K,N){(576,1536),(1536,576),(2048,5632),"
                                     "(4096,14336)}, quantise rows + GEMM + requant-LUT int8 out",
                            cold_l2="weight copies per shape > 3x L2, rotated every step",
                            parallelism=f"replicas x{world}"),
                roofline=roof, gpu_launches=launches, clocks=clk,
                per_shape_ms={f"{m}x{k}x{n}": round(t, 4) for (m, k, n), t in zip(shapes, per)},
                backend=comp.label)
    if rank == 0 and world == 1 and not args.no_e2e:
        line["e2e"] = e2e_gemm_sweep(comp, torch, args)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_sweep(threads=1)
    return line


def e2e_gemm_sweep(comp, torch, args):
    """Through the public API: per shape a pinned-host f32 A goes to the device,
    vgemmBlock runs (row quantise + GEMM with a resident weight), the int8
    output comes back to pinned host memory."""
    import numpy as np
    rng = np.random.default_rng(5)
    items = []
    h2d = d2h = 0
    for (m, k, n) in sweep_shapes():
        W = (rng.standard_normal((k, n), dtype=np.float32) * 0.02)
        w = comp.register_weight(W, k, n)
        A = torch.randn(m, k).pin_memory()
        items.append(dict(m=m, k=k, n=n, w=w, A=A, dA=torch.empty(m, k, device="cuda"),
                          out=torch.empty(m * n, dtype=torch.int8, device="cuda"),
                          hout=torch.empty(m * n, dtype=torch.int8).pin_memory()))
        h2d += 4 * m * k
        d2h += m * n

    def step():
        for it in items:
            it["dA"].copy_(it["A"], non_blocking=True)
            comp.vgemm_dev(it["dA"], it["m"], it["w"], 4, it["out"])
            it["hout"].copy_(it["out"], non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    comp.sync()
    ms = t0.elapsed_time(t1) / args.steps
    ops = sum(2.0 * m * k * n for (m, k, n) in sweep_shapes())
    return dict(value=ops / (ms / 1e3) / 1e12, unit="TOPS", h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                ms_per_step=ms, path="pinned H2D f32 A -> dc_vgemm (quantizeRows + GEMM, resident weight) -> D2H int8")


# ---- the reference's CPU path (oracle restatement) -----------------------------
def _cpu_shape_worker(args):
    """Time vgemmBlock's CPU path on one (K, N): quantizeCols of the whole weight
    (per call, as verified_core.js:430 does) and `rows` rows of quantizeRows +
    the LUT triple loop.  Returns (t_qcols, t_per_row)."""
    k, n, rows, seed = args
    import numpy as np
    import __graft_entry__ as G
    O = G.oracle()
    rng = np.random.default_rng(seed)
    W = rng.integers(-127, 128, k * n).astype(np.float32) * np.float32(0.01)
    A = rng.standard_normal(rows * k).astype(np.float32)
    t = time.perf_counter()
    wq, ws = O.quantize_cols(W, k, n)
    tq = time.perf_counter() - t
    t = time.perf_counter()
    xq, xs = O.quantize_rows(A, rows, k)
    O.bgemm(xq, wq, xs, ws, rows, k, n, 1, O.REQUANT)
    tr = (time.perf_counter() - t) / rows
    return tq, tr


def cpu_sweep_rate(threads: int, rows: int = 2):
    """Sweep throughput of the reference CPU algorithm, extrapolated from a
    bounded sample: per (K,N) one quantizeCols + `rows` LUT-GEMM rows."""
    jobs = [(k, n, rows, i) for i, (k, n) in enumerate(SWEEP_KN)]
    t0 = time.perf_counter()
    if threads > 1:
        import multiprocessing as mp
        with mp.get_context("spawn").Pool(min(threads, len(jobs))) as pool:
            res = pool.map(_cpu_shape_worker, jobs)
    else:
        res = [_cpu_shape_worker(j) for j in jobs]
    wall = time.perf_counter() - t0
    total_t = 0.0
    for (k, n), (tq, tr) in zip(SWEEP_KN, res):
        for m in SWEEP_M:
            total_t += tq + m * tr
    ops = sum(2.0 * m * k * n for (m, k, n) in sweep_shapes())
    return ops / total_t / 1e12, wall


def cpu_baseline_sweep(threads=1):
    v, wall = cpu_sweep_rate(threads)
    return dict(value=v, unit="TOPS", cores=threads, kind="port",
                sample=f"per (K,N): one per-call quantizeCols + 2 rows of quantizeRows + LUT GEMM "
                       f"(C restatement of verified_core.js, single thread), extrapolated to the 16 shapes; "
                       f"{wall:.1f} s of CPU work")


def bench_reference(args, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    vals = []
    for s in range(args.warmup + args.steps):
        # each step a bounded sample of the sweep spread over the host cores
        v, _ = cpu_sweep_rate(min(threads, len(SWEEP_KN)), rows=1)
        if s >= args.warmup:
            vals.append(v)
    v = statistics.median(vals)
    ops_step = sum(2.0 * m * k * n for (m, k, n) in sweep_shapes())
    ms = ops_step / (v * 1e12) * 1e3
    return dict(metric=METRIC, impl="reference", value=v, unit="TOPS (int8 ops/s, GEMM sweep)", n_gpus=world,
                steps=args.steps, warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling="weak",
                vs_baseline=None, dtype="int8 x int8 -> int32", data="synthetic (seeded)",
                config=dict(workload="gemm-sweep (same shapes)", parallelism="host cores"),
                cpu_baseline=dict(value=v, unit="TOPS", cores=min(threads, len(SWEEP_KN)), kind="port",
                                  sample="per (K,N): one per-call quantizeCols + 1 LUT-GEMM row per step, "
                                         "extrapolated; one process per (K,N)"),
                e2e=dict(value=v, unit="TOPS", h2d_bytes_per_step=0, d2h_bytes_per_step=0))


def traffic_for(key):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get(key)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemm-sweep", choices=["gemm-sweep"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    peaks = load_peaks()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = bench_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    rank, local, world = dist_init()
    line = bench_gemm_sweep(args, rank, world, peaks)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
