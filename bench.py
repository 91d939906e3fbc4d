#!/usr/bin/env python3
"""Benchmark of DaisyChain-Infer's verified INT8 W8A8 path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One JSON line (rank 0).  The metric is the reference's: INT8 decode tok/s and
chunked-prefill tok/s at 1/2/4/8 B200 (pipeline stages), with the GEMM's
fraction of the roofline.  Workloads (synthetic random-init models of the named
shapes; seeded uniform token ids; no dataset is involved):

* ``llama3-8b-chunked`` (default): hidden 4096, 32 layers, 32/8 heads, inter
  14336, vocab 128256, RoPE theta 500000; a 2048-token prompt prefilled in
  16-token chunks with two in flight, then 256 greedy decode tokens.  At N GPUs
  the 32 layers are split over N pipeline stages (planStages, equal capacity).
* ``tinyllama-chunked``: hidden 2048, 22 layers, 32/4 heads, inter 5632, vocab
  32000; 512-token prompt, chunks of 16, 128 decode tokens.
* ``smollm-135m-window``: hidden 576, 30 layers, 9/3 heads, inter 1536, vocab
  49152 (tied); full-window lookahead path, T = 64, 24-token prompt, 16 tokens.
* ``smollm-360m-lookahead``: hidden 960, 32 layers, 15/5 heads, inter 2560,
  vocab 49152 (tied); T = 512, a 256-token prompt of a seeded 8-gram repeated
  with 20% substitutions, 128 new tokens.
* ``gemm-sweep``: the standalone INT8 GEMM sweep (M in {1,16,128,512} x (K,N)).

One step = one whole generation (prefill + decode, or the lookahead laps).
``value`` is decode tokens/s (new tokens / decode time on the head);
``prefill_tok_s`` is prompt tokens / prefill time.  Timing: W untimed warm-up
steps, then K steps between barrier + synchronize, CUDA events on the launching
stream, max over ranks.  The model's weights (~8 GB for Llama-3-8B) exceed the
126 MB L2, so every step reads them from HBM.
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
MODEL_SEED = 20261201
SWEEP_M = [1, 16, 128, 512]
SWEEP_KN = [(576, 1536), (1536, 576), (2048, 5632), (4096, 14336)]
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    "llama3-8b-chunked": dict(spec=dict(hidden=4096, layers=32, heads=32, kvHeads=8, inter=14336, vocab=128256,
                                        ropeTheta=500000.0, tie=False),
                              mode="chunked", prompt=2048, new=256, chunk=16, window=2, per_pass=32,
                              name="Llama-3-8B-shaped decoder"),
    "tinyllama-chunked": dict(spec=dict(hidden=2048, layers=22, heads=32, kvHeads=4, inter=5632, vocab=32000,
                                        ropeTheta=10000.0, tie=False),
                              mode="chunked", prompt=512, new=128, chunk=16, window=2, per_pass=32,
                              name="TinyLlama-1.1B-shaped decoder"),
    "smollm-135m-window": dict(spec=dict(hidden=576, layers=30, heads=9, kvHeads=3, inter=1536, vocab=49152,
                                         ropeTheta=10000.0, tie=True),
                               mode="lookahead", prompt=24, new=16, T=64, name="SmolLM-135M-shaped decoder"),
    "smollm-360m-lookahead": dict(spec=dict(hidden=960, layers=32, heads=15, kvHeads=5, inter=2560, vocab=49152,
                                            ropeTheta=10000.0, tie=True),
                                  mode="lookahead", prompt="ngram", new=128, T=512,
                                  name="SmolLM-360M-shaped decoder"),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm_gbs=d["hbm_gbs"], bf16_tflops=d["bf16_tflops"],
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained"), src="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, src="fallback")


def traffic_for(key):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(key)
    return None


# ---- clocks during the timed region ----------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu, self.proc, self.path, self.t_start = gpu_index, None, None, 0.0

    def start(self):
        """Start sampling and wait (up to 10 s) for the first sample."""
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
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, local, world


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(vals, world):
    if world == 1:
        return list(vals)
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(vals), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def sum_over_ranks(vals, world):
    if world == 1:
        return list(vals)
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(vals), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


# ---- model workloads --------------------------------------------------------------------
def prompt_ids(w: dict, vocab: int, seed: int = 7):
    import numpy as np
    rng = np.random.default_rng(seed)
    if w["prompt"] == "ngram":
        gram = rng.integers(0, vocab, 8)
        ids = np.resize(gram, 256)
        sub = rng.random(256) < 0.2
        ids[sub] = rng.integers(0, vocab, int(sub.sum()))
        return [int(v) for v in ids]
    return [int(v) for v in rng.integers(0, vocab, w["prompt"])]


E2E_UNIT = "tok/s (prompt ids on the host to generated ids on the host, prefill included)"


def workload_config(name: str, world: int) -> dict:
    """The ``config`` object of both arms' lines (identical for the same
    workload and GPU count): the model shape, the schedule and the stages."""
    import __graft_entry__ as G
    shard = G.package().shard  # host logic only: no device call
    w = WORKLOADS[name]
    sp = w["spec"]
    n_prompt = 256 if w["prompt"] == "ngram" else w["prompt"]
    plan = shard.plan_stages(sp["layers"], [dict(id=f"gpu{i}", capacity=1.0) for i in range(world)])
    sched = (f"{n_prompt}-token prompt in chunks of {w['chunk']} ({w['window']} passes in flight, "
             f"{w['per_pass']} chunks per pass over the weights; ids identical to one chunk per pass), "
             f"{w['new']} greedy decode tokens" if w["mode"] == "chunked" else
             f"full-window lookahead T={w['T']}, {n_prompt}-token prompt, {w['new']} new tokens")
    return dict(workload=name, model=(f"{w['name']}: hidden {sp['hidden']}, {sp['layers']} layers, "
                                      f"{sp['heads']}/{sp['kvHeads']} heads, inter {sp['inter']}, vocab {sp['vocab']}"),
                schedule=sched, stages=[f"{s['lo']}-{s['hi']}" for s in plan], parallelism=f"pipeline x{world}",
                l2="weights >> L2: every step streams them from HBM")


def build_rank(P, comp, w: dict, rank: int, world: int):
    """This rank's stage of the plan (planStages over equal capacities)."""
    import torch
    spec = P.infer.Spec(**w["spec"])
    plan = P.shard.plan_stages(spec.layers, [dict(id=f"gpu{i}", capacity=1.0) for i in range(world)])
    assert len(plan) == world
    st = plan[rank]
    if w["mode"] == "chunked":
        max_rows, max_pos = max(w["chunk"] * w["per_pass"], 8), w["prompt"] + w["new"] + 1
    else:
        max_rows, max_pos = w["T"], w["T"]
    S = P.infer.Stage(comp, spec, st["lo"], st["hi"], head=(rank == 0), max_rows=max_rows, max_pos=max_pos)
    S.synth(MODEL_SEED, P.infer.SYNTH_FACTOR)
    dev = torch.device("cuda", comp.device)
    tp = P.pipeline.TorchP2P(P.pipeline.ring_edge_groups(world)) if world > 1 else None
    ring = P.pipeline.Ring(S, rank, world, spec.hidden, tp,
                           new_buffer=lambda n: torch.empty(n, dtype=torch.float32, device=dev))
    return spec, plan, S, ring


def P_fnv(ids):
    """FNV-1a of the generated ids (int32 little-endian): equal at every GPU count."""
    h = 0x811C9DC5
    for v in ids or []:
        for b in int(v).to_bytes(4, "little", signed=True):
            h = ((h ^ b) * 0x01000193) & 0xFFFFFFFF
    return h


def weight_bytes(spec, lo, hi, head):
    C, q, kv, I, V = spec.hidden, spec.heads * spec.headDim, spec.kvHeads * spec.headDim, spec.inter, spec.vocab
    per_layer = C * (q + 2 * kv) + q * C + 2 * C * I + I * C
    return (hi - lo) * per_layer + (C * V if head else 0)


def bench_model(args, rank, world, peaks):
    import torch
    import __graft_entry__ as G
    P = G.package()
    w = WORKLOADS[args.workload]
    comp = P.init_compute(int(os.environ.get("LOCAL_RANK", "0")), stream=torch.cuda.current_stream())
    spec, plan, S, ring = build_rank(P, comp, w, rank, world)
    ids = prompt_ids(w, spec.vocab)
    marks = {}

    def one_step():
        if w["mode"] == "chunked":
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            out = ring.generate_chunked(ids, w["new"], w["chunk"], w["window"], on_prefill=e1.record,
                                        per_pass=w["per_pass"])
            e2.record()
            marks.setdefault("ev", []).append((e0, e1, e2))
            return out
        e0, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = ring.generate_lookahead(ids, w["new"], w["T"], 4)
        e2.record()
        marks.setdefault("ev", []).append((e0, e0, e2))
        return out

    for _ in range(args.warmup):
        one_step()
    comp.sync()
    marks.clear()
    l0 = comp.L.dc_launch_count()
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    # (the GEMMs are timed in passes right after the timed region, which runs
    # with no per-GEMM events or stamps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    t0.record()
    outs = [one_step() for _ in range(args.steps)]
    t1.record()
    torch.cuda.nvtx.range_pop()
    gen_ids = None
    if rank == 0:
        o = outs[-1]
        gen_ids = [int(v) for v in (o.tolist() if hasattr(o, "tolist") else o[len(ids):])]
    torch.cuda.synchronize()
    clocks.mark_end()
    barrier(world)
    clk = clocks.stop()
    comp.sync()
    launches = comp.L.dc_launch_count() - l0
    ms_step = t0.elapsed_time(t1) / args.steps
    pre = statistics.mean(a.elapsed_time(b) for a, b, _ in marks["ev"])
    dec = statistics.mean(b.elapsed_time(c) for _, b, c in marks["ev"])
    # the GEMM timing of this rank: GEMV (decode) and tcgen05 (prefill)
    import ctypes as C

    def read_kinds():
        out = {}
        for kind in (1, 3):
            ms, n, by, op = C.c_double(), C.c_longlong(), C.c_double(), C.c_double()
            comp.L.dc_timing_read(comp.h, kind, C.byref(ms), C.byref(n), C.byref(by), C.byref(op))
            out[kind] = (ms.value, n.value, by.value, op.value)
        return out

    # one more generation with CUDA events around every GEMM launch (a chunked
    # workload: the same prompt and 16 decode tokens, decode laps launched
    # kernel by kernel; a lookahead workload: one more step)
    comp.L.dc_timing(comp.h, 1)
    if w["mode"] == "chunked":
        use_graph = getattr(ring, "use_graph", False)
        ring.use_graph = False
        ring.generate_chunked(ids, 16, w["chunk"], w["window"], per_pass=w["per_pass"])
        ring.use_graph = use_graph
        ev_scale = w["new"] * args.steps / 16.0
    else:
        one_step()
        ev_scale = args.steps
    got = read_kinds()
    comp.L.dc_timing(comp.h, 0)
    pre_wn = None
    if w["mode"] == "chunked" and world > 2:
        # labelled variant: as many passes in flight as there are stages (the
        # reference keeps two); the same ids
        pe = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(2):  # (the first run sizes the deeper hop-buffer rings)
            pe[0].record()
            ring.generate_chunked(ids, 1, w["chunk"], world, on_prefill=pe[1].record, per_pass=w["per_pass"])
        comp.sync()
        pre_wn = max_over_ranks([pe[0].elapsed_time(pe[1])], world)[0]
    pre1 = None
    if w["mode"] == "chunked" and w["per_pass"] > 1:
        # for comparison: the same prefill one chunk per pass over the weights
        pe = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(2):  # (the first run warms the one-chunk path)
            pe[0].record()
            ring.generate_chunked(ids, 1, w["chunk"], w["window"], on_prefill=pe[1].record, per_pass=1)
        comp.sync()
        pre1 = max_over_ranks([pe[0].elapsed_time(pe[1])], world)[0]
    tc_method = ("CUDA events around every tcgen05 launch of the same prompt's prefill, run right after the timed "
                 "region (launched one by one, as in the timed steps), times the timed steps")
    tl = None
    if w["mode"] == "chunked" and world == 1:
        # the timed decode laps are CUDA-graph replays: time their GEMVs inside
        # replays, from %globaltimer stamps between the launches of each lap
        tl = decode_timeline(S, ring, ids, w)
        laps = w["new"] * args.steps
        ops_per_byte = got[1][3] / got[1][2] if got[1][2] else 0.0
        gemv = (tl["gemv_ms_per_lap"] * laps, tl["gemv_launches_per_lap"] * laps,
                tl["gemv_bytes_per_lap"] * laps, tl["gemv_bytes_per_lap"] * laps * ops_per_byte)
        gemv_method = ("%%globaltimer stamps between the launches of %d CUDA-graph-replayed decode laps run right "
                       "after the timed region (dc_stage_set_timeline; same stages and shapes): a GEMV's time is "
                       "the gap from the stamp after the launch before it to the stamp after it, median over the "
                       "laps, times the timed region's laps; each gap includes one stamp launch (%.2f us, the "
                       "lap's growth per stamp)" % (tl["laps"], tl["stamp_cost_us"]))
    else:
        ms_, n_, by_, op_ = got[1]
        gemv = (ms_ * ev_scale, int(round(n_ * ev_scale)), by_ * ev_scale, op_ * ev_scale)
        gemv_method = ("CUDA events around every GEMV launch of the pass above (kernel by kernel), scaled to the "
                       "timed region's decode steps")
    kinds = {1: gemv, 3: tuple(v * args.steps for v in got[3])}
    ms_step, pre, dec = max_over_ranks([ms_step, pre, dec], world)
    launches = int(sum_over_ranks([launches], world)[0])
    n_new = w["new"]
    if w["mode"] == "lookahead":
        n_new = len(outs[-1]) - len(ids) if rank == 0 else w["new"]
    line = None
    if rank == 0:
        value = n_new / (dec / 1e3)
        dom = max(kinds, key=lambda k: kinds[k][0])
        ms, n, by, op = kinds[dom]
        per_launch_ms = ms / max(n, 1)
        ach = by / (ms / 1e3) / 1e9
        roof = dict(bound="hbm", achieved=ach, peak=peaks["hbm_gbs"], unit="GB/s", frac=ach / peaks["hbm_gbs"],
                    traffic=traffic_for("gemv_decode" if dom == 1 else "tc_prefill"),
                    kernel=("k_gemv_row (decode GEMV, M=1)" if dom == 1 else "k_gemm_tc (tcgen05, M>8)"),
                    launches=n, avg_launch_us=per_launch_ms * 1e3, share_of_step=ms / (ms_step * args.steps),
                    algorithmic_bytes_per_launch=by / max(n, 1), ops_per_launch=op / max(n, 1),
                    method=(gemv_method if dom == 1 else tc_method),
                    peak_source=f"{peaks['src']} HBM copy bandwidth (MEASURED_PEAKS.json)")
        other = {("gemv" if k == 1 else "tcgen05"): dict(ms=kinds[k][0], launches=kinds[k][1],
                                                          gbs=(kinds[k][2] / (kinds[k][0] / 1e3) / 1e9
                                                               if kinds[k][0] else None),
                                                          tops=(kinds[k][3] / (kinds[k][0] / 1e3) / 1e12
                                                                if kinds[k][0] else None))
                 for k in kinds}
        line = dict(metric=METRIC, value=value, unit="tok/s (decode)", n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=ms_step, higher_is_better=True, scaling="strong",
                    vs_baseline=None, dtype="int8 x int8 -> int32 (f32 epilogue, f64 norms/softmax)",
                    data="synthetic (random-init weights, seeded uniform token ids)",
                    config=workload_config(args.workload, world),
                    prefill_tok_s=(len(ids) / (pre / 1e3)) if w["mode"] == "chunked" else None,
                    prefill_ms=pre if w["mode"] == "chunked" else None, decode_ms=dec,
                    prefill_tok_s_one_chunk_per_pass=(len(ids) / (pre1 / 1e3)) if pre1 else None,
                    prefill_tok_s_window_n=(len(ids) / (pre_wn / 1e3)) if pre_wn else None,
                    roofline=roof, kernels=other, gpu_launches=launches, clocks=clk, backend=comp.label,
                    generated_ids_fnv=P_fnv(gen_ids), generated_head=gen_ids[:8],
                    weights_gb=weight_bytes(spec, 0, spec.layers, True) / 1e9)
        if tl is not None:
            line["decode_timeline"] = tl
    if not args.no_e2e:  # every rank takes part in the ring; rank 0 reports
        e2e = e2e_model(comp, ring, w, ids, args, world)
        if rank == 0:
            line["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_model_baseline(w)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    S.close()
    return line


def decode_timeline(S, ring, ids, w, laps: int = 17, per_lap: int = 2048):
    """Time the GEMVs of graph-replayed decode laps from the inside: one more
    generation of the same prompt with `laps` decode tokens, the head stage
    stamping %globaltimer after every launch of each lap (dc_stage_set_timeline).
    Lap 0 runs kernel by kernel (it is captured into the graph the others
    replay) and is dropped.  A GEMV's time is the gap between the stamp after it
    and the stamp after the launch before it; the figures are medians over the
    replayed laps.  The same generation without stamps gives the lap time the
    stamps are charged against."""
    import numpy as np
    import torch

    def decode_ms(stamped):
        buf = None
        if stamped:
            buf = torch.zeros(laps * per_lap, dtype=torch.int64, device="cuda")
            S.set_timeline(buf, per_lap, laps)
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        try:
            e[0].record()
            ring.generate_chunked(ids, laps, w["chunk"], w["window"], on_prefill=e[1].record,
                                  per_pass=w["per_pass"])
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            torch.cuda.synchronize()
            info = S.timeline_info() if stamped else None
        finally:
            if stamped:
                S.set_timeline()
        return e[1].elapsed_time(end), buf, info

    plain_ms, _, _ = decode_ms(False)
    stamped_ms, buf, (kinds, by) = decode_ms(True)
    n = len(kinds)
    if n < 2 or n > per_lap:
        raise RuntimeError(f"decode timeline: {n} stamps per lap (buffer holds {per_lap})")
    t = buf.view(laps, per_lap)[1:, :n].cpu().numpy().astype(np.float64)
    if not (t > 0).all():
        raise RuntimeError("decode timeline: a replayed lap left stamps unwritten")
    gaps = np.diff(t, axis=1) / 1e6  # ms; gaps[:, i - 1] is closed by stamp i
    k = np.asarray(kinds[1:])
    b = np.asarray(by[1:])
    gemv = k == 1
    lap_ms = np.median(t[:, -1] - t[:, 0]) / 1e6
    gemv_ms = float(np.median(gaps[:, gemv].sum(axis=1)))
    tc_ms = float(np.median(gaps[:, k == 3].sum(axis=1)))
    gemv_bytes = float(b[gemv].sum())
    per = gaps[:, gemv]
    # per GEMV shape: (bytes) -> median in-graph GB/s
    shapes = {}
    for col, bb in zip(range(per.shape[1]), b[gemv]):
        shapes.setdefault(round(bb), []).append(np.median(per[:, col]))
    stamp_cost_us = (stamped_ms - plain_ms) / laps / n * 1e3
    med = np.median(gaps, axis=0) * 1e3  # us, per launch of the lap
    # the layers' launch pattern: after the lap's first GEMV (lm_head of the
    # previous row) each layer has the same number of tagged GEMVs; the period
    # is the launches from one layer's first GEMV to the next layer's
    gp = [i for i, kk in enumerate(k) if kk == 1]
    nlay = max(1, S.hi - S.lo)
    layer_us, layer_kinds = None, None
    g_l = (len(gp) - 1) // nlay
    if g_l >= 1 and len(gp) > 1 + g_l:
        per_layer, start = gp[1 + g_l] - gp[1], gp[1] - 1
        nl = (len(med) - start) // per_layer
        if nl > 0:
            m = np.array([med[start + l * per_layer:start + (l + 1) * per_layer] for l in range(nl)])
            layer_us = [round(float(v), 2) for v in m.mean(axis=0)]
            layer_kinds = [int(v) for v in k[start:start + per_layer]]
    return dict(laps=laps - 1, stamps_per_lap=n, gemv_launches_per_lap=int(gemv.sum()),
                gemv_bytes_per_lap=gemv_bytes, gemv_ms_per_lap=gemv_ms,
                gemv_gbs=gemv_bytes / (gemv_ms / 1e3) / 1e9, tcgen05_ms_per_lap=tc_ms,
                stamped_lap_ms=float(lap_ms), plain_decode_ms_per_lap=plain_ms / laps,
                stamp_cost_us=stamp_cost_us,
                launch_us_first=[round(float(v), 2) for v in med[:21]],
                launch_us_last=[round(float(v), 2) for v in med[-8:]],
                launch_kinds_first=[int(v) for v in k[:21]], launch_kinds_last=[int(v) for v in k[-8:]],
                layer_us=layer_us, layer_kinds=layer_kinds,
                gemv_by_bytes_per_launch={str(kb): dict(launches_per_lap=len(v), us=float(np.median(v) * 1e3),
                                                        gbs=kb / (np.median(v) / 1e3) / 1e9)
                                          for kb, v in sorted(shapes.items())})


def e2e_model(comp, ring, w, ids, args, world=1):
    """Through the public API with host buffers: the prompt ids come from pinned
    host memory each step, the generated ids go back to host memory (on the
    head).  Every rank runs its part of the ring; the time is the max over
    ranks (the head's lap spans the others')."""
    import torch
    host_ids = torch.tensor(ids, dtype=torch.int32).pin_memory()
    steps = max(1, min(args.steps, 3))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = None
    barrier(world)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(steps):
        prompt = host_ids.tolist()
        if w["mode"] == "chunked":
            picks = ring.generate_chunked(prompt, w["new"], w["chunk"], w["window"], per_pass=w["per_pass"])
            out = picks.cpu() if picks is not None else None
        else:
            out = ring.generate_lookahead(prompt, w["new"], w["T"], 4)
    t1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks([t0.elapsed_time(t1) / steps], world)[0]
    n_new = w["new"]
    return dict(value=n_new / (ms / 1e3), unit=E2E_UNIT,
                h2d_bytes_per_step=4 * len(ids), d2h_bytes_per_step=4 * n_new, ms_per_step=ms,
                path="host ids -> infer/pipeline API (embed, stages, logits, greedy) -> host ids")


# ---- the reference's CPU path (oracle restatement), sampled ----------------------------
def cpu_model_rates(w: dict):
    """Time the reference's CPU algorithm on a bounded sample of the workload:
    one layer of this model (vgemmBlock re-quantising every weight per call, as
    verified_core.js:430 does) for one decode row, one 16-row prefill chunk (or
    one full window), and lm_head over 1/16 of the vocabulary, then
    extrapolate linearly to all layers and the whole vocabulary."""
    import numpy as np
    import __graft_entry__ as G
    O = G.oracle()
    sp = w["spec"]
    spec = O.Spec(hidden=sp["hidden"], layers=1, heads=sp["heads"], kvHeads=sp["kvHeads"], inter=sp["inter"],
                  vocab=max(16, sp["vocab"] // 16), ropeTheta=sp["ropeTheta"], tie=False)
    C_, q, kv, I_ = spec.hidden, spec.heads * spec.headDim, spec.kvHeads * spec.headDim, spec.inter
    s = MODEL_SEED
    wts = {"emb": O.synth_weight(s, -1, "emb", spec.vocab, C_), "nrmF": np.ones(C_, np.float32),
           "lm": O.synth_weight(s, -1, "lm", C_, spec.vocab),
           "layers": [dict(nrm1=np.ones(C_, np.float32), nrm2=np.ones(C_, np.float32),
                           Wq=O.synth_weight(s, 0, "Wq", C_, q), Wk=O.synth_weight(s, 0, "Wk", C_, kv),
                           Wv=O.synth_weight(s, 0, "Wv", C_, kv), Wo=O.synth_weight(s, 0, "Wo", q, C_),
                           Wgate=O.synth_weight(s, 0, "Wgate", C_, I_), Wup=O.synth_weight(s, 0, "Wup", C_, I_),
                           Wdown=O.synth_weight(s, 0, "Wdown", I_, C_))]}
    m = O.Model(spec, wts, per_call_quant=True)
    rng = np.random.default_rng(1)
    out = {}
    if w["mode"] == "chunked":
        kvc = O.KV(m, 0, 1, 64)
        x = m.embed_rows(rng.integers(0, spec.vocab, 16))
        t = time.perf_counter()
        y = m.run_layers(x, 0, 1, kvc, 0)
        out["chunk_layer_s"] = time.perf_counter() - t
        t = time.perf_counter()
        m.run_layers(m.embed_rows([3]), 0, 1, kvc, 16)
        out["decode_layer_s"] = time.perf_counter() - t
        t = time.perf_counter()
        m.logits_rows(y, [15])
        out["lm_sample_s"] = time.perf_counter() - t
        L, V16 = sp["layers"], 16
        out["decode_tok_s"] = 1.0 / (L * out["decode_layer_s"] + V16 * out["lm_sample_s"])
        out["prefill_tok_s"] = 16.0 / (L * out["chunk_layer_s"])
    else:
        T = w["T"]
        x = m.embed_rows(rng.integers(0, spec.vocab, T))
        t = time.perf_counter()
        y = m.run_layers(x, 0, 1)
        out["window_layer_s"] = time.perf_counter() - t
        t = time.perf_counter()
        m.logits_rows(y, [T - 1])
        out["lm_sample_s"] = time.perf_counter() - t
        out["decode_tok_s"] = 1.0 / (sp["layers"] * out["window_layer_s"] + 16 * out["lm_sample_s"])
    return out


def cpu_threads():
    import __graft_entry__ as G
    return G.oracle().threads()


def cpu_e2e_rate(w: dict, r: dict):
    """Whole-generation rate (prefill included) of the sampled CPU rates."""
    n_prompt = 256 if w["prompt"] == "ngram" else w["prompt"]
    if "prefill_tok_s" not in r:  # the full-window path: every token is one lap
        return r["decode_tok_s"]
    return w["new"] / (n_prompt / r["prefill_tok_s"] + w["new"] / r["decode_tok_s"])


SAMPLE_DESC = ("one layer of this model through the C restatement of verified_core.js/infer.js (weights re-quantised "
               "per call as vgemmBlock does, LUT GEMM) for one decode row and one 16-row chunk (or one full window), "
               "plus lm_head over 1/16 of the vocabulary; extrapolated to every layer and the whole vocabulary")


def cpu_model_baseline(w, samples: int = 3):
    t = time.perf_counter()
    rs = [cpu_model_rates(w) for _ in range(samples)]
    wall = time.perf_counter() - t
    cores = cpu_threads()
    med = {k: statistics.median(r[k] for r in rs) for k in rs[0]}
    return dict(value=med["decode_tok_s"], unit="tok/s (decode)", cores=cores, kind="port",
                prefill_tok_s=med.get("prefill_tok_s"), e2e_tok_s=cpu_e2e_rate(w, med),
                sample=f"{SAMPLE_DESC}; median of {samples} samples, {wall:.1f} s of CPU work on {cores} threads "
                       "(GEMMs and quantisers split by output element; the reference's own JS path uses one)",
                detail=med)


def bench_reference(args, rank, world):
    """The reference's CPU implementation of the path, timed on this host."""
    if rank != 0:
        return None
    if args.workload == "gemm-sweep":
        for _ in range(args.warmup):
            cpu_sweep_rate()
        res = [cpu_sweep_rate() for _ in range(max(1, args.steps))]
        v = statistics.median(r[0] for r in res)
        ms = statistics.mean(r[1] for r in res) * 1e3
        unit = "TOPS (int8 ops/s, GEMM sweep)"
        extra = {}
    else:
        # one step = one bounded sample of the workload (one layer, one decode
        # row, one chunk or window, 1/16 of lm_head); the model-level rates are
        # the median of the steps' extrapolations
        w = WORKLOADS[args.workload]
        for _ in range(args.warmup):
            cpu_model_rates(w)
        walls, rs = [], []
        for _ in range(args.steps):
            t = time.perf_counter()
            rs.append(cpu_model_rates(w))
            walls.append((time.perf_counter() - t) * 1e3)
        med = {k: statistics.median(r[k] for r in rs) for k in rs[0]}
        v = med["decode_tok_s"]
        ms = statistics.mean(walls)
        unit = "tok/s (decode)"
        e2e_v = cpu_e2e_rate(w, med)
        extra = dict(prefill_tok_s=med.get("prefill_tok_s"),
                     extrapolated=dict(decode_tok_s=v, prefill_tok_s=med.get("prefill_tok_s"), e2e_tok_s=e2e_v,
                                       method="each step times the sample; its rates are extrapolated to every layer "
                                              "and the whole vocabulary; value is the median over the steps"),
                     config=workload_config(args.workload, world))
        sample = SAMPLE_DESC
        return dict(metric=METRIC, impl="reference", value=v, unit=unit, n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling="strong", vs_baseline=None,
                    dtype="int8 x int8 -> int32 (f32 epilogue, f64 norms/softmax)",
                    data="synthetic (random-init weights, seeded uniform token ids)",
                    cpu_baseline=dict(value=v, unit=unit, cores=cpu_threads(), kind="port", sample=sample),
                    e2e=dict(value=e2e_v, unit=E2E_UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0,
                             path="the sampled CPU rates combined over the whole generation (prefill included)"),
                    **extra)
    sample = "per (K,N): one per-call quantizeCols + 2 LUT-GEMM rows, extrapolated to the 16 shapes"
    return dict(metric=METRIC, impl="reference", value=v, unit=unit, n_gpus=world, steps=args.steps,
                warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling="weak", vs_baseline=None,
                dtype="int8 x int8 -> int32", data="synthetic (seeded)", config=sweep_config(world),
                cpu_baseline=dict(value=v, unit=unit, cores=cpu_threads(), kind="port", sample=sample),
                e2e=dict(value=v, unit=unit, h2d_bytes_per_step=0, d2h_bytes_per_step=0), **extra)


# ---- the GEMM sweep -----------------------------------------------------------------
def sweep_config(world: int) -> dict:
    return dict(workload="gemm-sweep", shapes="M in {1,16,128,512} x (K,N) in {(576,1536),(1536,576),(2048,5632),"
                "(4096,14336)}", cold_l2="weight copies per shape > 3x L2, rotated", parallelism=f"replicas x{world}")


def sweep_shapes():
    return [(m, k, n) for (k, n) in SWEEP_KN for m in SWEEP_M]


def _cpu_shape_worker(args):
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
    return tq, (time.perf_counter() - t) / rows


def cpu_sweep_rate(rows: int = 2):
    jobs = [(k, n, rows, i) for i, (k, n) in enumerate(SWEEP_KN)]
    t0 = time.perf_counter()
    res = [_cpu_shape_worker(j) for j in jobs]
    wall = time.perf_counter() - t0
    total_t = sum(tq + m * tr for (k, n), (tq, tr) in zip(SWEEP_KN, res) for m in SWEEP_M)
    ops = sum(2.0 * m * k * n for (m, k, n) in sweep_shapes())
    return ops / total_t / 1e12, wall


def int8_reference_peak(peaks):
    """Dense int8 peak for the tensor-bound shapes: cuBLASLt's int8 GEMM
    (torch._int_mm, int32 out) at 8192^3, best of 10, measured here; 2 x the
    measured bf16 figure when that call is unavailable."""
    import torch
    try:
        a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1)
            best = t if best is None else min(best, t)
        return 2.0 * 8192 ** 3 / (best / 1e3) / 1e12, "measured cuBLASLt int8 GEMM (torch._int_mm 8192^3, best of 10)"
    except Exception as ex:  # noqa: BLE001
        return 2.0 * peaks["bf16_tflops"], f"2 x measured bf16 dense TFLOP/s (torch._int_mm unavailable: {ex})"[:160]


def bench_gemm_sweep(args, rank, world, peaks):
    """The standalone GEMM sweep.  Each shape's GEMM launches (rotating over
    weight copies whose total exceeds 3x the L2, so every launch reads its
    weights from HBM) are captured once in a CUDA graph; one step replays every
    shape's graph, each bracketed by CUDA events, so the device times are
    kernel times, not host launch latency."""
    import torch
    import __graft_entry__ as G
    P = G.package()
    comp = P.init_compute(int(os.environ.get("LOCAL_RANK", "0")), stream=torch.cuda.current_stream())
    g = torch.Generator(device="cuda").manual_seed(2026)
    items = []
    for (m, k, n) in sweep_shapes():
        ld = (k + 15) // 16 * 16
        copies = min(512, max(3, math.ceil(3 * L2_BYTES / (n * ld))))
        W = torch.randint(-127, 128, (copies, n, ld), generator=g, device="cuda", dtype=torch.int8)
        if ld != k:
            W[:, :, k:] = 0
        it = dict(m=m, k=k, n=n, ld=ld, W=W, copies=copies,
                  cs=torch.rand(copies, n, generator=g, device="cuda") * 9e-3 + 1e-3,
                  xq=torch.zeros(m, ld, dtype=torch.int8, device="cuda"), rs=torch.empty(m, device="cuda"),
                  out=torch.empty(m * n, dtype=torch.int8, device="cuda"))
        A = torch.randn(m, k, generator=g, device="cuda")
        comp.quantize_rows_dev(A, m, k, it["xq"], ld, it["rs"])
        items.append(it)

    def launch(it, c):
        comp.bgemm_dev(it["xq"], it["ld"], it["W"][c], it["ld"], it["rs"], it["cs"][c], it["m"], it["k"], it["n"],
                       1, 4, it["out"])

    for it in items:  # warm-up outside capture (tensor maps, shared-memory limits, split-K scratch)
        for c in range(min(it["copies"], 3)):
            launch(it, c)
    comp.sync()
    cap = torch.cuda.Stream()
    for it in items:
        graph = torch.cuda.CUDAGraph()
        comp.set_stream(cap)  # outside the capture: switching streams synchronises the old one
        with torch.cuda.graph(graph, stream=cap):
            for c in range(it["copies"]):
                launch(it, c)
        comp.set_stream(torch.cuda.current_stream())
        it["graph"] = graph
    launches_per_step = sum(it["copies"] for it in items)

    def step(evs=None):
        for i, it in enumerate(items):
            if evs is not None:
                evs[i][0].record()
            it["graph"].replay()
            if evs is not None:
                evs[i][1].record()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    shape_ev = []
    t0.record()
    for s in range(args.steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in items]
        step(evs)
        shape_ev.append(evs)
    t1.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    barrier(world)
    clk = clocks.stop()
    comp.sync()
    i8_peak, i8_src = int8_reference_peak(peaks)
    shapes = []
    for i, it in enumerate(items):
        us = statistics.mean(ev[i][0].elapsed_time(ev[i][1]) for ev in shape_ev) * 1e3 / it["copies"]
        m, k, n = it["m"], it["k"], it["n"]
        byts = m * k + k * n + 4 * m + 4 * n + m * n
        ops = 2.0 * m * k * n
        gbs, tops = byts / us / 1e3, ops / us / 1e6
        tensor_bound = ops / byts * peaks["hbm_gbs"] / 1e3 > i8_peak  # AI x BW above the int8 peak
        frac = tops / i8_peak if tensor_bound else gbs / peaks["hbm_gbs"]
        shapes.append(dict(m=m, k=k, n=n, us=round(us, 2), gbs=round(gbs, 1), tops=round(tops, 1),
                           bound="tensor" if tensor_bound else "hbm", frac=round(frac, 3),
                           kernel="k_gemv_row" if m == 1 else ("k_gemv" if m <= 8 else "k_gemm_tc"),
                           launches_per_replay=it["copies"]))
    ms = max_over_ranks([t0.elapsed_time(t1) / args.steps], world)[0]
    ops_step = sum(2.0 * it["m"] * it["k"] * it["n"] * it["copies"] for it in items)
    # the dominant kernel: the tcgen05 GEMM at the largest tensor-bound shape
    top = max((s for s in shapes if s["bound"] == "tensor"), key=lambda s: s["m"] * s["k"] * s["n"])
    roof = dict(bound="tensor", achieved=top["tops"], peak=i8_peak, unit="TOPS", frac=top["tops"] / i8_peak,
                traffic=traffic_for("tc_m512"), kernel=f"k_gemm_tc at M={top['m']} K={top['k']} N={top['n']}",
                method="CUDA events around a graph replay of this shape's launches (weight copies > 3x L2)",
                peak_source=i8_src)
    line = None
    if rank == 0:
        line = dict(metric=METRIC, value=ops_step * world / (ms / 1e3) / 1e12, unit="TOPS (int8 ops/s, GEMM sweep)",
                    n_gpus=world, steps=args.steps, warmup=args.warmup, ms_per_step=ms, higher_is_better=True,
                    scaling="weak", vs_baseline=None, dtype="int8 x int8 -> int32", data="synthetic (seeded)",
                    config=sweep_config(world), roofline=roof, gpu_launches=launches_per_step * args.steps,
                    clocks=clk, backend=comp.label, per_shape=shapes, int8_peak_tops=i8_peak,
                    int8_peak_source=i8_src)
        if world == 1 and not args.no_cpu:
            v, wall = cpu_sweep_rate()
            line["cpu_baseline"] = dict(value=v, unit="TOPS", cores=cpu_threads(), kind="port",
                                        sample=f"per (K,N): one per-call quantizeCols + 2 LUT-GEMM rows, "
                                               f"extrapolated; {wall:.1f} s")
    return line


def profile_gemm(args):
    """One GEMM of the sweep inside an NVTX range "profile", for an ncu capture
    of exactly that launch (M = --gemm-m, K = --gemm-k, N = --gemm-n, requant
    int8 out), after three warm-up calls of the same shape:

        ncu --set full --nvtx --nvtx-include "profile/" -k regex:k_gemm ... python bench.py --profile gemm"""
    import torch
    import __graft_entry__ as G
    P = G.package()
    comp = P.init_compute(0, stream=torch.cuda.current_stream())
    m, k, n = args.gemm_m, args.gemm_k, args.gemm_n
    g = torch.Generator(device="cuda").manual_seed(1)
    W = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    cs = torch.rand(n, generator=g, device="cuda") * 9e-3 + 1e-3
    xq = torch.zeros(m, k, dtype=torch.int8, device="cuda")
    rs = torch.empty(m, device="cuda")
    comp.quantize_rows_dev(torch.randn(m, k, generator=g, device="cuda"), m, k, xq, k, rs)
    out = torch.empty(m * n, dtype=torch.int8, device="cuda")
    for _ in range(3):
        comp.bgemm_dev(xq, k, W, k, rs, cs, m, k, n, 1, 4, out)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profile")
    comp.bgemm_dev(xq, k, W, k, rs, cs, m, k, n, 1, 4, out)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    comp.sync()
    return dict(profiled="gemm", m=m, k=k, n=n, flags="requant int8")


def profile_model(args):
    """One prefill pass or one decode lap of the workload, inside an NVTX range
    named "profile", for an ncu launch list of exactly that unit of work:

        ncu --nvtx --nvtx-include "profile/" --metrics gpu__time_duration.sum ...
            python bench.py --profile decode

    The prompt is prefilled first (outside the range), so the profiled chunk or
    lap sees the full-length KV cache of the benchmark.  Prints what it ran."""
    import torch
    import __graft_entry__ as G
    P = G.package()
    w = WORKLOADS[args.workload]
    assert w["mode"] == "chunked", "--profile takes a chunked workload"
    comp = P.init_compute(0, stream=torch.cuda.current_stream())
    spec, plan, S, ring = build_rank(P, comp, w, 0, 1)
    ids = prompt_ids(w, spec.vocab)
    chunks = P.shard.prefill_chunks(len(ids), w["chunk"], w["window"])["chunks"]
    passes = P.shard.chunk_passes(chunks, w["per_pass"])
    S.kv_reset()
    last = None
    for i, (lo, hi, rows) in enumerate(passes):
        inside = args.profile == "prefill" and i == len(passes) - 1
        if inside:
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("profile")
        last = P.infer.run_ring([S], S.embed_rows(ids[lo:hi]), lo, rows)
        if inside:
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
    if args.profile == "decode":
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("profile")
        S.decode_many([S], last, 1, use_graph=False)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    comp.sync()
    S.close()
    return dict(profiled=args.profile, workload=args.workload, prompt=len(ids),
                unit=("the last prefill pass (rows %d..%d, %d chunks)" % (passes[-1][0], passes[-1][1],
                                                                         len(passes[-1][2]))
                      if args.profile == "prefill" else "one decode lap at KV length %d" % len(ids)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama3-8b-chunked", choices=list(WORKLOADS) + ["gemm-sweep"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--prompt-len", type=int, default=0, help="override the prompt length (profiling runs)")
    ap.add_argument("--new-tokens", type=int, default=0, help="override the generated tokens (profiling runs)")
    ap.add_argument("--per-pass", type=int, default=0, help="override the chunks per pass over the weights")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (profiling runs)")
    ap.add_argument("--profile", choices=["prefill", "decode", "gemm"], default=None,
                    help="run one prefill chunk, one decode lap or one sweep GEMM inside an NVTX range 'profile' "
                         "(for ncu); prints no benchmark line")
    ap.add_argument("--gemm-m", type=int, default=512, help="M of the --profile gemm launch")
    ap.add_argument("--gemm-k", type=int, default=4096, help="K of the --profile gemm launch")
    ap.add_argument("--gemm-n", type=int, default=14336, help="N of the --profile gemm launch")
    args = ap.parse_args()
    if args.workload in WORKLOADS:
        w = WORKLOADS[args.workload]
        if args.prompt_len and w["prompt"] != "ngram":
            w["prompt"] = args.prompt_len
        if args.new_tokens:
            w["new"] = args.new_tokens
        if args.per_pass and w["mode"] == "chunked":
            w["per_pass"] = args.per_pass
        if args.layers:
            w["spec"] = dict(w["spec"], layers=args.layers)
    args.warmup = max(args.warmup, 3)
    peaks = load_peaks()
    if args.profile:
        print(json.dumps(profile_gemm(args) if args.profile == "gemm" else profile_model(args)), flush=True)
        return
    if args.impl == "reference":
        line = bench_reference(args, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    rank, local, world = dist_init()
    if args.workload == "gemm-sweep":
        line = bench_gemm_sweep(args, rank, world, peaks)
    else:
        line = bench_model(args, rank, world, peaks)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
