#!/usr/bin/env python
"""Benchmark of the streaming-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the multi-head GQA decode sweep at its
largest point): one decode step of attention for batch 1, 16 query heads
sharing 8 KV heads, head_dim 128, KV length T = 262144, fp32 (the reference's
element type), block 64, scale 1/sqrt(128); Q/K/V i.i.d. N(0,1) from a fixed
seed.  K+V = 2 GiB > L2 (126 MB), so every timed step streams from HBM with
no flush needed.

A step = one pass of the hot path over that sequence.  At N = 1 one
sa_attn_decode launch.  At N > 1 (torchrun, one rank per GPU) the sequence is
split evenly over the ranks (strong scaling, configs[1]'s "KV sequence split
evenly over 1/2/4/8 GPUs"): each rank runs one sa_attn_decode_sp launch over
its T/N rows, whose merging CTAs exchange the per-head (m, l, O) states over
NVLink and merge them -- the sequence-parallel decomposition of
streaming_attention_mpi_simple.  The weak-scaling figure (T rows on every
GPU) is reported beside it.

Metric: attention GB/s = algorithmic bytes (K + V + q + out, each read or
written once) / time, whole job.  `e2e` is the same metric through the C ABI
with pinned HOST buffers for the step's inputs and output.  `roofline`
compares the decode kernel's own time with the measured HBM copy bandwidth.
`graph` repeats the step as 100 calls replayed from one CUDA graph (median of
5).  `cpu_baseline` and `--impl reference` time the reference's own CPU
implementation (streaming_attention_omp per query head, compiled from the
reference's sources into oracle/_ref/libsa_ref.so) on the host cores with an
explicit thread count.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HQ, HKV, D, T_GLOBAL, BLOCK = 16, 8, 128, 262144, 64
GRAPH_CALLS = 100          # calls per CUDA-graph replay of the graph measurement
SCALE = 1.0 / math.sqrt(D)
SEED = 20261201
METRIC = "attn GB/s"
WORKLOAD = ("configs[1] GQA decode: B=1, hq=16, hkv=8, d=128, T=262144 split evenly over the GPUs, "
            "block 64, scale 1/sqrt(128), fp32, N(0,1) seeded")
FALLBACK_HBM_GBS = 6650.0


def algo_bytes(T: int, elt: int = 4) -> int:
    return (2 * HKV * T * D + 2 * HQ * D) * elt


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock / throttle reasons while work runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            f = [x.strip() for x in r.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- helpers
def load_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic(key: str):
    """DRAM bytes per launch from a committed ncu summary (profiles/ncu_traffic.txt)."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        for line in open(p):
            f = line.split()
            if len(f) >= 2 and f[0] == key:
                return float(f[1])
    except OSError:
        pass
    return None


def make_inputs(T: int, dtype, device, seed: int):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(HQ, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    k = torch.randn(HKV, T, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    v = torch.randn(HKV, T, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    return q, k, v


def make_slice(T_total: int, t0: int, T: int, device, seed: int):
    """q and rows [t0, t0 + T) of K and V of one seeded T_total-row sequence
    (every rank generates the same sequence and keeps its slice)."""
    import torch
    q, k, v = make_inputs(T_total, torch.float32, device, seed)
    if t0 == 0 and T == T_total:
        return q, k, v
    ks, vs = k[:, t0:t0 + T].contiguous(), v[:, t0:t0 + T].contiguous()
    del k, v
    return q, ks, vs


def cpu_reference_time(q, k, v, T_sample: int, budget_s: float, min_reps: int = 3):
    """Time the reference CPU path (per-head streaming_attention_omp, all host
    threads) on a T_sample-row slice of the workload; returns (s per
    step-of-sample, reps, threads)."""
    from oracle.oracle import Reference
    import numpy as np
    R = Reference()
    cores = host_cores()
    ks = np.ascontiguousarray(k[:, :T_sample])
    vs = np.ascontiguousarray(v[:, :T_sample])
    out = np.empty((HQ, D), np.float32)
    R.gqa_decode_omp(q, ks, vs, BLOCK, cores, SCALE, out)       # warm-up (page-in, threads)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        R.gqa_decode_omp(q, ks, vs, BLOCK, cores, SCALE, out)
        times.append(time.perf_counter() - t0)
        if len(times) >= 1000:
            break
    return statistics.median(times), len(times), cores


# ---------------------------------------------------------------- reference arm
def host_cores() -> int:
    """Host threads this process may run on (torchrun does not restrict the
    affinity, but it sets OMP_NUM_THREADS=1, so the count is passed to the
    reference explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def decode_config(world: int) -> dict:
    """The workload both arms report (identical dicts, so the two lines pair up)."""
    return {"workload": WORKLOAD, "kv_len": T_GLOBAL, "kv_split": world,
            "T_per_gpu": T_GLOBAL // world,
            "parallelism": f"sp{world}" if world > 1 else "single",
            "l2": "inputs (2 GiB K+V in total) exceed L2 (126 MB); no flush"}


def make_inputs_np(T: int, seed: int):
    """Host copy of the global sequence: the values the GPU arm generates (on
    the GPU's generator when there is one)."""
    import torch
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    q, k, v = make_inputs(T, torch.float32, dev, seed)
    return q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()


def run_reference(args):
    """--impl reference: the reference's streaming_attention_omp per query head
    (attention/src/streaming_omp.cpp:99-154, compiled from its sources) over
    the whole T_GLOBAL-row sequence, every step, with all host threads."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    import numpy as np
    from oracle.oracle import Reference
    q, k, v = make_inputs_np(T_GLOBAL, SEED)
    R = Reference()
    cores = host_cores()
    out = np.empty((HQ, D), np.float32)
    for _ in range(args.warmup):
        R.gqa_decode_omp(q, k, v, BLOCK, cores, SCALE, out)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        R.gqa_decode_omp(q, k, v, BLOCK, cores, SCALE, out)
    el = time.perf_counter() - t0
    gbs = algo_bytes(T_GLOBAL) * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": decode_config(args.gpus),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": f"streaming_attention_omp per query head (16) over all {T_GLOBAL} rows "
                                   f"per step, num_threads={cores} passed explicitly"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
        return 2
    if T_GLOBAL % (world * 64):
        print(f"bench.py: T={T_GLOBAL} does not split into {world} x 64-row shares", file=sys.stderr)
        return 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # gloo carries only the exchange-buffer handles, barriers and the max
        # over ranks of the timings; the attention exchange is the kernel's own
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))

    import streaming_attention_b200 as sa
    from streaming_attention_b200 import _capi
    from streaming_attention_b200.sequence_parallel import SpDecoder
    ctx = sa.Context(local)
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)
    L = _capi.lib()
    sp = None
    if world > 1:
        sp = SpDecoder(ctx, rank, world, max_hq=HQ, max_d=D)
        sp.connect_dist()

    T = T_GLOBAL // world
    # rank r holds rows [r*T, (r+1)*T) of one seeded global sequence
    q, k, v = make_slice(T_GLOBAL, rank * T, T, dev, SEED)
    out = torch.empty(HQ, D, device=dev)
    P = lambda t: _capi.C.c_void_p(t.data_ptr()) if t is not None else None

    def decode_once(q_, k_, v_, T_, out_):
        if world == 1:
            _capi.check(L.sa_attn_decode(ctx.h, 0, P(q_), P(k_), P(v_), T_ * D, T_, D, HQ, HKV, BLOCK,
                                         SCALE, P(out_), 0))
        else:
            _capi.check(L.sa_attn_decode_sp(sp.h, 0, P(q_), P(k_), P(v_), T_ * D, T_, D, HQ, HKV, BLOCK,
                                            SCALE, P(out_), None, None, 0))

    step = lambda: decode_once(q, k, v, T, out)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def tmax(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up, then a ~1 s soak under clock sampling that runs into the timed region
    for _ in range(args.warmup):
        step()
    barrier()
    if args.profile:
        # short device-only sequence for ncu: W warm-up launches + K launches
        for _ in range(args.steps):
            step()
        barrier()
        if rank == 0:
            print(json.dumps({"profile": True, "launches": args.warmup + args.steps}), flush=True)
        if sp:
            sp.close()
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        return 0
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    smi_id = vis.split(",")[local].strip() if vis else str(local)
    clocks = ClockSampler(smi_id)
    clocks.start()
    s0 = time.perf_counter()
    while tmax(time.perf_counter() - s0) < 1.0:   # one decision for all ranks: same step count everywhere
        for _ in range(50):
            step()
        torch.cuda.synchronize(dev)
    barrier()

    # timed region: K steps, CUDA events on the launching stream, max over ranks
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = tmax(ev0.elapsed_time(ev1))
    ms_step = ms / args.steps
    value = algo_bytes(T_GLOBAL) * args.steps / (ms / 1e3) / 1e9

    # the same step as GRAPH_CALLS calls replayed from one CUDA graph, median of 5
    graph, g_ms, graph_err = None, [], None
    try:
        gs = torch.cuda.Stream(dev)
        ctx.set_stream(gs.cuda_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=gs):
            for _ in range(GRAPH_CALLS):
                step()
        graph = g
    except Exception as e:          # reported, never required
        graph_err = str(e)
    ctx.set_stream(stream.cuda_stream)
    # replay only if every rank captured (a rank alone would wait for the others)
    if -tmax(-(1.0 if graph is not None else 0.0)) > 0:
        for _ in range(2):
            graph.replay()
        for _ in range(5):
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cur = torch.cuda.current_stream(dev)
            e0.record(cur)
            graph.replay()
            e1.record(cur)
            torch.cuda.synchronize(dev)
            g_ms.append(tmax(e0.elapsed_time(e1)) / GRAPH_CALLS)
    elif graph_err is None:
        graph_err = "another rank could not capture the step"
    barrier()

    # kernel-only timing for the roofline: this rank's decode launches back to back
    # (at N > 1 the same fused launch: slice + exchange + merge)
    kt0 = torch.cuda.Event(enable_timing=True)
    kt1 = torch.cuda.Event(enable_timing=True)
    nk = max(20, args.steps)
    barrier()
    kt0.record(stream)
    for _ in range(nk):
        step()
    kt1.record(stream)
    torch.cuda.synchronize(dev)
    k_ms = tmax(kt0.elapsed_time(kt1) / nk)

    result = None
    if rank == 0:
        peak, peak_kind = load_peak()
        achieved = algo_bytes(T) / (k_ms / 1e3) / 1e9
        traffic = load_traffic("decode_f32_T262144")
        if traffic is not None and world > 1:
            traffic = traffic / world      # DRAM bytes scale with the rows a launch streams
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": decode_config(world),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"{peak_kind} hbm_gbs (copy bandwidth)",
                         "per": "GPU (this rank's slice: K + V + q + out bytes / launch time)",
                         "kernel": "sa::dec::decode_kernel<float,128,2>" +
                                   (" with the sequence-parallel exchange" if world > 1 else ""),
                         "kernel_ms": round(k_ms, 5), "traffic": traffic},
            "clocks": clk,
            "gpu_launches": args.steps,
            "gpu_launches_per": "rank (one launch per step per rank)",
        }
        if g_ms:
            med = statistics.median(g_ms)
            result["graph"] = {"calls": GRAPH_CALLS, "repeats": 5, "ms_per_step_median": round(med, 5),
                               "value_median": round(algo_bytes(T_GLOBAL) / (med / 1e3) / 1e9, 2),
                               "ms_per_step_all": [round(x, 5) for x in g_ms]}
        else:
            result["graph"] = {"error": graph_err}
    if graph is not None:
        del graph

    # ---- e2e through the C ABI with pinned host buffers
    hq_ = q.cpu().pin_memory()
    hout = torch.empty(HQ, D).pin_memory()
    HP = lambda t: _capi.C.c_void_p(t.data_ptr())
    ne = max(3, min(args.steps, 20))
    # the new token's key/value rows, appended at the last row of the sequence
    # (which the last rank holds) every step
    hkn = k[:, T - 1].cpu().pin_memory()
    hvn = v[:, T - 1].cpu().pin_memory()

    def e2e_step():
        if world == 1:
            # one decode step through the C ABI: host q / k_new / v_new in, the
            # KV cache resident in HBM, host output back (sa_attn_decode_step)
            _capi.check(L.sa_attn_decode_step(ctx.h, 0, HP(hq_), HP(hkn), HP(hvn), P(k), P(v), T,
                                              T - 1, D, HQ, HKV, BLOCK, SCALE, HP(hout),
                                              _capi.SA_HOST_PTRS))
        else:
            # the same step sharded: q from pinned host memory on every rank,
            # the new row appended by the last rank, one fused launch per rank,
            # the output read back
            with torch.cuda.stream(stream):
                q.copy_(hq_, non_blocking=True)
                if rank == world - 1:
                    k[:, T - 1].copy_(hkn, non_blocking=True)
                    v[:, T - 1].copy_(hvn, non_blocking=True)
            step()
            with torch.cuda.stream(stream):
                hout.copy_(out, non_blocking=True)
            stream.synchronize()

    for _ in range(2):
        e2e_step()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    w0 = time.perf_counter()
    for _ in range(ne):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - w0
    e_ms = tmax(max(e0.elapsed_time(e1), wall * 1e3))
    e2e = algo_bytes(T_GLOBAL) * ne / (e_ms / 1e3) / 1e9

    # the attention.h drop-in with every K/V byte copied from host memory per
    # call (PCIe-bound by construction), reported beside e2e
    e2e_kv = None
    if world == 1:
        hk = k.cpu().pin_memory()
        hv = v.cpu().pin_memory()
        nh = 3
        _capi.check(L.sa_attn_decode(ctx.h, 0, HP(hq_), HP(hk), HP(hv), T * D, T, D, HQ, HKV, BLOCK,
                                     SCALE, HP(hout), _capi.SA_HOST_PTRS))
        h0 = torch.cuda.Event(enable_timing=True)
        h1 = torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for _ in range(nh):
            _capi.check(L.sa_attn_decode(ctx.h, 0, HP(hq_), HP(hk), HP(hv), T * D, T, D, HQ, HKV,
                                         BLOCK, SCALE, HP(hout), _capi.SA_HOST_PTRS))
        h1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_kv = algo_bytes(T) * nh / (h0.elapsed_time(h1) / 1e3) / 1e9
        del hk, hv

    # ---- weak scaling (extra): T_GLOBAL rows on EVERY GPU, the same fused step
    weak = None
    if world > 1 and not args.no_extra:
        del q, k, v
        torch.cuda.empty_cache()
        qw, kw, vw = make_slice(T_GLOBAL * world, rank * T_GLOBAL, T_GLOBAL, dev, SEED)
        wstep = lambda: decode_once(qw, kw, vw, T_GLOBAL, out)
        for _ in range(args.warmup):
            wstep()
        barrier()
        w0e, w1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0e.record(stream)
        for _ in range(args.steps):
            wstep()
        w1e.record(stream)
        barrier()
        wms = tmax(w0e.elapsed_time(w1e))
        weak = {"value": round(algo_bytes(T_GLOBAL) * world * args.steps / (wms / 1e3) / 1e9, 2),
                "unit": "GB/s", "ms_per_step": round(wms / args.steps, 5), "kv_len": T_GLOBAL * world,
                "T_per_gpu": T_GLOBAL, "scaling": "weak"}

    if rank == 0:
        if world == 1:
            result["e2e"] = {"value": round(e2e, 2), "unit": "GB/s",
                             "h2d_bytes_per_step": (HQ * D + 2 * HKV * D) * 4,
                             "d2h_bytes_per_step": HQ * D * 4, "steps": ne,
                             "path": "sa_attn_decode_step(SA_HOST_PTRS): q and the new token's k/v "
                                     "from pinned host memory appended to the HBM-resident KV "
                                     "cache, attention over all T rows, output read back"}
            result["e2e_host_kv"] = {
                "value": round(e2e_kv, 2), "unit": "GB/s",
                "h2d_bytes_per_step": (HQ * D + 2 * HKV * T * D) * 4,
                "d2h_bytes_per_step": HQ * D * 4,
                "path": "sa_attn_decode(SA_HOST_PTRS): all of q, K, V copied from pinned host "
                        "memory every call (attention.h drop-in; PCIe-bound)"}
        else:
            result["e2e"] = {"value": round(e2e, 2), "unit": "GB/s",
                             "h2d_bytes_per_step": (HQ * D + 2 * HKV * D) * 4,
                             "d2h_bytes_per_step": HQ * D * 4, "steps": ne,
                             "path": "decode step over the sharded HBM-resident KV cache: q from pinned "
                                     "host memory on every rank, the new token's k/v appended by the "
                                     "last rank, sa_attn_decode_sp (one launch per rank, exchange over "
                                     "NVLink), output read back"}
            if weak:
                result["weak_scaling"] = weak
        # ---- CPU baseline: the reference's CPU path on a bounded sample (rank 0, N=1)
        if world == 1 and not args.no_cpu:
            try:
                qn, kn, vn = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
                T_s = 65536
                t_s, reps, cores = cpu_reference_time(qn, kn, vn, T_s, budget_s=args.cpu_budget)
                result["cpu_baseline"] = {
                    "value": round(algo_bytes(T_s) / t_s / 1e9, 3), "unit": "GB/s",
                    "cores": cores, "kind": "reference",
                    "sample": f"streaming_attention_omp per query head (16 heads) over the first "
                              f"{T_s} of {T_GLOBAL} KV rows, {reps} reps, median, num_threads={cores}"}
            except Exception as e:  # the baseline is reported, never required
                result["cpu_baseline"] = {"value": None, "unit": "GB/s", "cores": host_cores(),
                                          "kind": "reference", "sample": f"unavailable: {e}"}
        if world == 1 and not args.no_extra:
            pms, ptf = measure_prefill(ctx, dev, stream, 10, 3)
            bpk, bkind = load_bf16_peak()
            result["extra"] = {"prefill_configs2": {
                "metric": "attn TFLOP/s (causal prefill)", "value": round(ptf, 2),
                "ms": round(pms, 4), "frac_of_bf16_peak": round(ptf / bpk, 4),
                "peak": f"{bpk} ({bkind} bf16_tflops)", "workload": PF_WORKLOAD}}
            try:
                q3, weights = measure_qwen3(ctx, dev, stream, 20, 3, long_prompt=True)
                q3line = {"metric": "Qwen3-0.6B tok/s", "workload": Q3_WORKLOAD,
                          **{k_: round(v_, 4) for k_, v_ in q3.items()}}
                q3line["roofline"] = qwen3_roofline(q3)
                if not args.no_cpu:
                    try:
                        q3line["cpu_baseline"] = cpu_qwen3_baseline(weights)
                    except Exception as e:
                        q3line["cpu_baseline"] = {"value": None, "sample": f"unavailable: {e}"}
                result["extra"]["qwen3_configs3_4"] = q3line
            except Exception as e:
                result["extra"]["qwen3_configs3_4"] = {"error": str(e)}
        print(json.dumps(result), flush=True)

    if sp:
        sp.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------- prefill
PF_S, PF_HQ, PF_HKV = 8192, 16, 8
PF_WORKLOAD = ("configs[2] causal prefill: Q [8192, 16, 128], K/V [8192, 8, 128] bf16 N(0,1), "
               "scale 1/sqrt(128), fp32 accumulation")


def prefill_flops(S=PF_S, hq=PF_HQ, d=D):
    """Causal FLOPs: 2 GEMMs x 2 FLOP x hq x d x S(S+1)/2 (the non-causal 2x is not counted)."""
    return 4.0 * hq * d * S * (S + 1) / 2


def measure_prefill(ctx, dev, stream, steps, warmup, out_dtype="bfloat16"):
    import torch
    import streaming_attention_b200 as sa
    g = torch.Generator(device=dev).manual_seed(SEED)
    q = torch.randn(PF_S, PF_HQ, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(PF_S, PF_HKV, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(PF_S, PF_HKV, D, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(PF_S, PF_HQ, D, device=dev, dtype=getattr(torch, out_dtype))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)    # 256 MB > L2
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            sa.attn_prefill(q, k, v, SCALE, 0, out_dtype, ctx, out)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tot = 0.0
        for _ in range(steps):
            flush.zero_()                       # L2 flush between timed launches
            e0.record(stream)
            sa.attn_prefill(q, k, v, SCALE, 0, out_dtype, ctx, out)
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
    ms = tot / steps
    return ms, prefill_flops() / (ms / 1e3) / 1e12


def load_bf16_peak(sustained=False):
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["bf16_tflops_sustained" if sustained else "bf16_tflops"]), "measured"
    except Exception:
        return (1400.0 if sustained else 1590.0), "fallback"


def cpu_prefill_baseline(budget_s: float, reps: int = 1):
    """The reference's ops::self_attention_streaming_blockwise_avx2 (ops.cpp:1453-1524,
    q/kv blocks 128 as its driver uses) on the configs[2] head layout at a sample
    sequence length sized to about budget_s / 3 per call; returns the cpu_baseline dict."""
    import numpy as np
    from oracle.oracle import Reference
    R = Reference()
    rng = np.random.default_rng(SEED)

    def inputs(S):
        return (rng.standard_normal((S, PF_HQ, D), dtype=np.float32),
                rng.standard_normal((S, PF_HKV, D), dtype=np.float32),
                rng.standard_normal((S, PF_HKV, D), dtype=np.float32))

    q, k, v = inputs(1024)
    t0 = time.perf_counter()
    R.causal_prefill(q, k, v, SCALE, 128, 128, avx2=True)
    t1 = time.perf_counter() - t0
    S = int(min(PF_S, max(1024, 1024 * (max(budget_s, 1.0) / 3 / max(t1, 1e-3)) ** 0.5)) // 128 * 128)
    q, k, v = inputs(S)
    t0 = time.perf_counter()
    for _ in range(reps):
        R.causal_prefill(q, k, v, SCALE, 128, 128, avx2=True)
    el = (time.perf_counter() - t0) / reps
    tf = prefill_flops(S) / el / 1e12
    cores = os.cpu_count() or 1
    return {"value": round(tf, 5), "unit": "TFLOP/s", "cores": cores, "kind": "reference",
            "sample": f"self_attention_streaming_blockwise_avx2 (q/kv blocks 128), S={S} of {PF_S}, "
                      f"{PF_HQ}/{PF_HKV} heads, d {D}, {el:.2f} s per call, {cores} OpenMP threads"}


def run_prefill_reference(args):
    """--impl reference for the prefill workload: the reference's AVX2 block-wise
    causal prefill on the host cores, each step a bounded sample."""
    if env_int("RANK", 0) != 0:
        return 0
    per_step = max(2.0, 90.0 / (args.steps + args.warmup))
    cb = cpu_prefill_baseline(per_step * 3, reps=max(1, args.steps))
    print(json.dumps({
        "impl": "reference", "metric": "attn TFLOP/s (causal prefill)", "value": cb["value"],
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(prefill_flops() / (cb["value"] * 1e12) * 1e3, 3) if cb["value"] else None,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": PF_WORKLOAD, "parallelism": "cpu"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def run_prefill_sp(args):
    """configs[2] on N GPUs: zig-zag sequence-parallel causal prefill through
    sa_spp_prefill (each rank two query chunks; its K/V chunks stored into every
    rank's buffer over NVLink; one tensor-core launch over key-block pieces and
    their log-sum-exp merge).  Total work is fixed (strong scaling); time = max
    over ranks of CUDA-event time per step."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import SpPrefill, zigzag_shard
    world, rank, local = env_int("WORLD_SIZE", 1), env_int("RANK", 0), env_int("LOCAL_RANK", 0)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    g = torch.Generator(device=dev).manual_seed(SEED)     # the same full tensors on every rank
    q = torch.randn(PF_S, PF_HQ, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(PF_S, PF_HKV, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(PF_S, PF_HKV, D, device=dev, generator=g).to(torch.bfloat16)
    ql, kl, vl = zigzag_shard(q, rank, world), zigzag_shard(k, rank, world), zigzag_shard(v, rank, world)
    del q, k, v
    ctx = sa.Context(local)
    sp = SpPrefill(ctx, rank, world, max_seq=PF_S, hkv=PF_HKV)
    sp.connect_dist()
    out = torch.empty(ql.shape, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    main = torch.cuda.Stream(dev)

    with torch.cuda.stream(main):
        for _ in range(args.warmup):
            sp.prefill(ql, kl, vl, SCALE, out)
    torch.cuda.synchronize(dev)
    dist.barrier(device_ids=[local])
    tot = 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.steps):
        with torch.cuda.stream(main):
            flush.zero_()
            dist.barrier(device_ids=[local])
            e0.record(main)
            sp.prefill(ql, kl, vl, SCALE, out)
            e1.record(main)
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    t = torch.tensor([tot / args.steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tf = prefill_flops() / (ms / 1e3) / 1e12
    if rank == 0:
        peak, kind = load_bf16_peak()
        print(json.dumps({
            "metric": "attn TFLOP/s (causal prefill)", "value": round(tf, 2), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": PF_WORKLOAD, "parallelism": f"sp{world} zig-zag (2 chunks/rank, K/V "
                                                             "stored to every rank over NVLink, key-block "
                                                             "pieces merged by log-sum-exp)",
                       "l2": "256 MB buffer written between timed steps"},
            "roofline": {"bound": "tensor", "achieved": round(tf / world, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / world / peak, 4), "per": "GPU",
                         "peak_kind": f"{kind} bf16_tflops (burst)"},
            "gpu_launches": 4 * args.steps}), flush=True)
    ctx.synchronize()
    sp.close()
    ctx.close()
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    return 0


def run_prefill(args):
    import torch
    import streaming_attention_b200 as sa
    if env_int("WORLD_SIZE", 1) > 1:
        return run_prefill_sp(args)
    local = env_int("LOCAL_RANK", 0)
    if env_int("RANK", 0) != 0:
        return 0
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = sa.Context(local)
    stream = torch.cuda.Stream(dev)
    if args.profile:
        g = torch.Generator(device=dev).manual_seed(SEED)
        q = torch.randn(PF_S, PF_HQ, D, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(PF_S, PF_HKV, D, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(PF_S, PF_HKV, D, device=dev, generator=g).to(torch.bfloat16)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup + args.steps):
                sa.attn_prefill(q, k, v, SCALE, 0, "bfloat16", ctx)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile": True, "workload": "prefill",
                          "launches": args.warmup + args.steps}), flush=True)
        return 0
    clocks = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local].strip()
                          if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local))
    clocks.start()
    ms, tf = measure_prefill(ctx, dev, stream, args.steps, args.warmup)
    clk = clocks.stop()
    peak, kind = load_bf16_peak()
    cpu = None
    if not args.no_cpu:
        try:
            cpu = cpu_prefill_baseline(args.cpu_budget)
        except Exception as e:    # the reference build is optional on the box
            cpu = {"value": None, "unit": "TFLOP/s", "sample": f"unavailable: {e}"}
    print(json.dumps({
        "metric": "attn TFLOP/s (causal prefill)", "value": round(tf, 2), "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": PF_WORKLOAD, "l2": "256 MB buffer written between timed launches"},
        "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tf / peak, 4), "peak_kind": f"{kind} bf16_tflops (burst)",
                     "kernel": "sa::pf::prefill_kernel", "kernel_ms": round(ms, 4),
                     "traffic": load_traffic("prefill_S8192")},
        "cpu_baseline": cpu,
        "clocks": clk, "gpu_launches": args.steps}), flush=True)
    ctx.close()
    return 0


# ---------------------------------------------------------------- Qwen3
Q3_PROMPT, Q3_GEN = 128, 100
Q3_WORKLOAD = ("configs[3]/[4] Qwen3-0.6B random-init (bf16-exact N(0,0.02) weights, tied lm_head), "
               "batch 1: prefill of a 128-token prompt (logits for all positions, as qwen3_forward); "
               "decode of 100 greedy tokens after a 128-token prompt with the KV cache")


def measure_qwen3(ctx, dev, stream, steps, warmup, weights=None, long_prompt=False, rank=0, world=1,
                  strategy="head"):
    """Returns dict with prefill / decode tok/s (device-resident and e2e).
    With world > 1 every rank runs its head-parallel share (sa_qwen3_create_tp)
    of the same calls; each timed region starts after a barrier and its time
    is the maximum over the ranks."""
    import ctypes as C
    import torch
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import _capi
    cfg = sa.QWEN3_0_6B
    if weights is None:
        weights = sa.qwen3.random_weights(cfg, SEED)
    max_seq = 4096 + Q3_GEN + 8 if long_prompt else 512
    m = sa.Qwen3(cfg, max_seq=max_seq, ctx=ctx, rank=rank, world=world, strategy=strategy)
    m.load(weights)

    def sync():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def tmax(v):
        if world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if world > 1:
        m.connect()
    L = _capi.lib()
    rng = __import__("numpy").random.default_rng(SEED)
    ids = rng.integers(0, cfg["vocab"], Q3_PROMPT).astype("int64")
    ids_d = torch.from_numpy(ids).to(dev)
    logits_d = torch.empty(Q3_PROMPT, cfg["vocab"], device=dev)
    P = lambda t: C.c_void_p(t.data_ptr())
    out = {}
    with torch.cuda.stream(stream):
        ctx.set_stream(stream.cuda_stream)
        # ---- prefill, inputs resident (device ids -> device logits)
        def pf():
            _capi.check(L.sa_qwen3_forward(m.h, C.cast(P(ids_d), C.POINTER(C.c_int64)), Q3_PROMPT, 0,
                                           C.cast(P(logits_d), C.POINTER(C.c_float)), 0, 0))
        for _ in range(warmup):
            pf()
        stream.synchronize()
        sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            pf()
        e1.record(stream)
        e1.synchronize()
        pms = tmax(e0.elapsed_time(e1) / steps)
        out["prefill_tok_s"] = Q3_PROMPT / (pms / 1e3)
        out["prefill_ms"] = pms
        # ---- prefill e2e: pinned host ids in, pinned host logits [128, V] out,
        # through the C ABI with SA_HOST_PTRS (blocking call)
        ids_h = torch.from_numpy(ids).pin_memory()
        logits_h = torch.empty(Q3_PROMPT, cfg["vocab"]).pin_memory()
        def pf_host():
            _capi.check(L.sa_qwen3_forward(m.h, C.cast(P(ids_h), C.POINTER(C.c_int64)), Q3_PROMPT, 0,
                                           C.cast(P(logits_h), C.POINTER(C.c_float)), 0,
                                           _capi.SA_HOST_PTRS))
        pf_host()
        sync()
        t0 = time.perf_counter()
        ne = max(2, min(steps, 5))
        for _ in range(ne):
            pf_host()
        out["prefill_e2e_tok_s"] = Q3_PROMPT * ne / tmax(time.perf_counter() - t0)
        if long_prompt:
            # configs[4]'s second run: the 4096-token prompt (cache-free, last-token logits)
            ids_l = torch.from_numpy(rng.integers(0, cfg["vocab"], 4096).astype("int64")).to(dev)
            last_d = torch.empty(1, cfg["vocab"], device=dev)
            def pf_long():
                _capi.check(L.sa_qwen3_forward(m.h, C.cast(P(ids_l), C.POINTER(C.c_int64)), 4096, 0,
                                               C.cast(P(last_d), C.POINTER(C.c_float)), 1, 0))
            for _ in range(2):
                pf_long()
            stream.synchronize()
            sync()
            e0.record(stream)
            for _ in range(3):
                pf_long()
            e1.record(stream)
            e1.synchronize()
            lms = tmax(e0.elapsed_time(e1) / 3)
            out["prefill_4096_ms"] = lms
            out["prefill_4096_tok_s"] = 4096 / (lms / 1e3)
        # ---- decode: generate(101) - generate(1) = 100 decode steps (same prefill)
        def gen(n, prompt):
            m.reset()
            sync()
            t0 = time.perf_counter()
            toks = m.generate(prompt, n)
            return tmax(time.perf_counter() - t0), toks
        for p_len, key in ([(Q3_PROMPT, "decode")] + ([(4096, "decode_4096")] if long_prompt else [])):
            prompt = rng.integers(0, cfg["vocab"], p_len).astype("int64")
            gen(Q3_GEN + 1, prompt)                       # warm-up
            reps = 3
            t_long = min(gen(Q3_GEN + 1, prompt)[0] for _ in range(reps))
            t_short = min(gen(1, prompt)[0] for _ in range(reps))
            dt = max(t_long - t_short, 1e-9)
            out[f"{key}_tok_s"] = Q3_GEN / dt
            out[f"{key}_ms_per_token"] = dt / Q3_GEN * 1e3
    m.close()
    return out, weights


def qwen3_bytes_flops(S: int = Q3_PROMPT):
    """Algorithmic weight bytes of one Qwen3-0.6B pass (bf16: every layer
    matrix and the tied embedding / lm_head once) and the FLOPs of an S-token
    prefill (2 per weight per token + causal attention)."""
    import streaming_attention_b200 as sa
    c = sa.QWEN3_0_6B
    H, D_, I, V = c["hidden"], c["head_dim"], c["inter"], c["vocab"]
    QD, KD = c["hq"] * D_, c["hkv"] * D_
    layer = QD * H + 2 * KD * H + H * QD + 3 * I * H
    params = c["n_layers"] * layer + V * H
    attn = c["n_layers"] * 4 * c["hq"] * D_ * S * (S + 1) / 2
    return params * 2, 2.0 * S * params + attn


def qwen3_roofline(res: dict) -> dict:
    """Roofline of the Qwen3 measurements (HBM-bound: the weights are read once
    per pass).  Decode adds the KV cache read of its mean context at bf16
    width (the algorithmic minimum; the cache here is fp32, so the fraction is
    conservative)."""
    import streaming_attention_b200 as sa
    c = sa.QWEN3_0_6B
    peak, kind = load_peak()
    wbytes, flops = qwen3_bytes_flops()
    kv_row = c["n_layers"] * 2 * c["hkv"] * c["head_dim"] * 2          # bytes per cached token
    out = {"bound": "hbm", "peak": peak, "unit": "GB/s", "peak_kind": f"{kind} hbm_gbs",
           "weight_bytes": wbytes}
    if "prefill_ms" in res:
        t = res["prefill_ms"] / 1e3
        out["prefill"] = {"bytes": wbytes, "flops": flops, "ms": round(res["prefill_ms"], 4),
                          "achieved": round(wbytes / t / 1e9, 1), "frac": round(wbytes / t / 1e9 / peak, 4)}
    if "prefill_4096_ms" in res:
        # 4096 tokens: compute-bound (2 FLOP per weight per token + causal attention)
        f4 = qwen3_bytes_flops(4096)[1]
        tpk, tkind = load_bf16_peak()
        tf = f4 / (res["prefill_4096_ms"] / 1e3) / 1e12
        out["prefill_4096"] = {"bound": "tensor", "flops": f4, "ms": round(res["prefill_4096_ms"], 3),
                               "achieved_tflops": round(tf, 1), "peak_tflops": tpk,
                               "frac": round(tf / tpk, 4), "peak_kind": f"{tkind} bf16_tflops (burst)"}
    for key, ctx0 in (("decode", Q3_PROMPT), ("decode_4096", 4096)):
        ms = res.get(f"{key}_ms_per_token")
        if ms:
            b = wbytes + kv_row * (ctx0 + Q3_GEN / 2)
            out[key] = {"bytes_per_token": int(b), "ms_per_token": round(ms, 4),
                        "achieved": round(b / (ms / 1e3) / 1e9, 1), "frac": round(b / (ms / 1e3) / 1e9 / peak, 4)}
    return out


def cpu_qwen3_baseline(weights, budget_tokens=16):
    """The reference's AVX2 Qwen3 forward (qwen3_ops_avx.cpp:383) on the host:
    prefill of a bounded prompt, and a few cached decode steps."""
    import numpy as np
    from oracle.oracle import Qwen3Cfg, Reference
    import streaming_attention_b200 as sa
    c = sa.QWEN3_0_6B
    cfg = Qwen3Cfg(**{k: c[k] for k in ("vocab", "hidden", "n_layers", "hq", "hkv", "head_dim", "inter",
                                        "eps", "theta")})
    R = Reference()
    m = R.qwen3(cfg, weights)
    ids = np.random.default_rng(SEED).integers(0, cfg.vocab, budget_tokens).astype(np.int64)
    t0 = time.perf_counter()
    m.forward(ids, method=1)
    t_pf = time.perf_counter() - t0
    kv = m.new_cache(budget_tokens + 8)
    m.forward_cached(kv, ids, method=1)
    steps = 3
    t0 = time.perf_counter()
    nxt = 0
    for _ in range(steps):
        lg = m.forward_cached(kv, np.array([nxt], np.int64), method=1)
        nxt = int(np.argmax(lg[-1]))
    t_dec = time.perf_counter() - t0
    m.free_cache(kv)
    m.close()
    return {"value": round(budget_tokens / t_pf, 3), "unit": "tok/s",
            "prefill_tok_s": budget_tokens / t_pf, "decode_tok_s": steps / t_dec,
            "cores": os.cpu_count(), "kind": "reference",
            "sample": f"avx2::qwen3_forward_avx on a {budget_tokens}-token prompt; "
                      f"{steps} cached decode steps (qwen3_forward_avx_with_cache) after it; "
                      f"{os.cpu_count()} OpenMP threads"}


def run_qwen3_reference(args):
    """--impl reference for the qwen3 workload: the reference's AVX2 Qwen3-0.6B
    forward on the host cores with the same random-init weights (bounded prompt)."""
    if env_int("RANK", 0) != 0:
        return 0
    import streaming_attention_b200 as sa
    weights = sa.qwen3.random_weights(sa.QWEN3_0_6B, SEED)
    cb = cpu_qwen3_baseline(weights)
    print(json.dumps({
        "impl": "reference", "metric": "Qwen3-0.6B tok/s (prefill)", "value": cb["value"], "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(Q3_PROMPT / cb["prefill_tok_s"] * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": Q3_WORKLOAD, "parallelism": "cpu"},
        "decode": {"decode_tok_s": round(cb["decode_tok_s"], 3)},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def run_qwen3(args):
    import torch
    import streaming_attention_b200 as sa
    local, rank, world = env_int("LOCAL_RANK", 0), env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    if world > 1:
        # head-parallel over the ranks; gloo carries only the exchange-buffer
        # handles, barriers and the max over ranks of each timing
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    elif rank != 0:
        return 0
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = sa.Context(local)
    stream = torch.cuda.Stream(dev)
    if args.profile:
        # short sequence for ncu: one cache-free 128-token forward, then a
        # generate of 4 tokens (prefill + 3 captured decode steps)
        import numpy as np
        cfg = sa.QWEN3_0_6B
        m = sa.Qwen3(cfg, max_seq=4096 + 64 if args.long_prompt else 512, ctx=ctx)
        m.load(sa.qwen3.random_weights(cfg, SEED))
        ids = np.random.default_rng(SEED).integers(0, cfg["vocab"], Q3_PROMPT)
        m.forward(ids, logits="all")
        m.generate(ids, 4)
        if args.long_prompt:   # one 4096-token forward (tensor-core prompt attention)
            m.reset()
            m.forward(np.random.default_rng(SEED).integers(0, cfg["vocab"], 4096), logits="last")
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile": True, "workload": "qwen3"}), flush=True)
        return 0
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local].strip() if vis else str(local))
    clocks.start()
    res, weights = measure_qwen3(ctx, dev, stream, args.steps, args.warmup, long_prompt=args.long_prompt,
                                 rank=rank, world=world, strategy=args.strategy)
    clk = clocks.stop()
    if rank != 0:
        ctx.close()
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
        return 0
    line = {
        "metric": "Qwen3-0.6B tok/s (prefill)", "value": round(res["prefill_tok_s"], 1), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["prefill_ms"], 4), "higher_is_better": True,
        "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None, "dtype": "bf16 weights, fp32 activations", "data": "synthetic",
        "config": {"workload": Q3_WORKLOAD,
                   "parallelism": "single" if world == 1 else
                   (f"head-parallel over {world} GPUs" if args.strategy == "head" else
                    f"sequence-parallel over {world} GPUs (prompt tokens split, decode replicated)")},
        "decode": {k: round(v, 3) for k, v in res.items() if k.startswith("decode")},
        "e2e": {"value": round(res["prefill_e2e_tok_s"], 1), "unit": "tok/s",
                "h2d_bytes_per_step": Q3_PROMPT * 8, "d2h_bytes_per_step": Q3_PROMPT * 151936 * 4},
        "clocks": clk,
    }
    rl = qwen3_roofline(res)
    line["roofline"] = {"bound": "hbm", "achieved": rl["prefill"]["achieved"], "peak": rl["peak"], "unit": "GB/s",
                        "frac": rl["prefill"]["frac"], "traffic": None,
                        "per": "whole forward (weight bytes of one pass / prefill time)", "detail": rl}
    if not args.no_cpu and world == 1:
        try:
            line["cpu_baseline"] = cpu_qwen3_baseline(weights)
        except Exception as e:
            line["cpu_baseline"] = {"value": None, "sample": f"unavailable: {e}"}
    print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--long-prompt", action="store_true",
                    help="qwen3 workload: also decode after a 4096-token prompt (configs[4] second run)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the extra (non-headline) measurements in the decode line")
    ap.add_argument("--workload", choices=["decode", "prefill", "qwen3"], default="decode",
                    help="decode: the headline configs[1] line; prefill: configs[2] causal "
                         "prefill on tensor cores (TFLOP/s)")
    ap.add_argument("--profile", action="store_true",
                    help="only W warm-up + K device steps (a short launch sequence for ncu)")
    ap.add_argument("--strategy", choices=["head", "sequence"], default="head",
                    help="qwen3 workload on N > 1 GPUs: head-parallel or sequence-parallel")
    ap.add_argument("--cpu-budget", type=float, default=10.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "prefill":
        return run_prefill_reference(args) if args.impl == "reference" else run_prefill(args)
    if args.workload == "qwen3":
        return run_qwen3_reference(args) if args.impl == "reference" else run_qwen3(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
