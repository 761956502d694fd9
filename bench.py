"""Benchmark of the INT8 weight-only MatMul path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one step): the decode GEMV set at GPT-2-small shapes -- QKV 768x2304,
attn-out 768x768, FFN-up 768x3072, FFN-down 3072x768, LM head 768x50257 (tied),
each at M = 1 and M = 8 token rows (10 independent MatMulQ problems, run as one
mtrtq_gemv_group launch; --step-launch calls: one launch each), fp32 activations ~ N(0,1),
int8 per-channel weights from N(0, 0.02), MTRTQ_MODE_FP32 (activations keep the
reference's fp32 values; --mode bf16 rounds them once). Every call has 6
device copies of its weights and consecutive steps rotate through them (548 MB
of int8 weights in all, > 4x the 126 MB L2), so weights stream from HBM. The
calls are launched with MTRTQ_OPT_OVERLAP_LAUNCH (each may start while the one
ahead finishes; --no-overlap turns it off).

metric/value: algorithmic bytes (int8 W + scales + fp32 X + fp32 Y) per second
over the whole job, inputs resident in HBM, steps replayed as CUDA graphs, timed
with CUDA events on the launching stream. e2e: the same bytes per second through
the C ABI called from the host with pinned host buffers, host->device copy of
each call's activations and device->host copy of each output inside the timed
region. Secondary lines: the prefill tensor-core GEMM (TFLOP/s) at the large
shapes, and the single-op FFN-up case.

Multi-GPU (torchrun, one process per GPU): the same decode GEMV set strong-scaled
over the ranks (each call's output channels split per rank, one grouped launch of
the shards, one all-gather of the outputs through peer memory by the library's
own kernels); value = the set's bytes per step x steps / the max over ranks of
the timed region. --multi replicas: each rank its own full set (weak scaling);
that figure is also kept in the sharded line's method.replicas.

--impl reference: the reference's own CPU MatMulQ (oracle/_ref, compiled from
its sources) on the same workload, every call split into row x column-chunk
pieces (rows and columns are independent in its loop), each prepared once and
timed as the kernel call alone, spread over all host threads; rank 0 only. It
imports nothing of the package (inputs come from workloads.py loaded by path).
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

METRIC = "int8-W GEMM TFLOP/s & GEMV HBM GB/s vs peak; GPT-2 decode tok/s @1/2/4/8 GPU"
UNIT = "GB/s"
WEIGHT_COPIES = 6
DECODE_SET_WORKLOAD = ("decode GEMV set, GPT-2-small shapes (QKV 768x2304, attn-out 768x768, FFN-up 768x3072, "
                       "FFN-down 3072x768, LM head 768x50257) x M in {1,8}")
DECODE_SET_WEIGHT_BYTES = 2 * (768 * 2304 + 768 * 768 + 768 * 3072 + 3072 * 768 + 768 * 50257)  # M = 1 and 8
E2E_STREAMS = 3  # host-buffer calls of a step spread over this many streams
LAUNCHES_PER_GRAPH = 4 * WEIGHT_COPIES  # dominant-kernel timing: launches per graph
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["bf16", "fp32"], default="fp32",
                    help="fp32 (default): activations keep the reference's fp32 values; bf16: rounded once")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--workload", default="decode_set",
                    help="decode_set (default), shape:M,K,N (one MatMulQ shape timed alone), gpt2_decode, "
                         "tp_decode (GPT-2-XL tensor parallel over the ranks) or sharded:M,K,N,S")
    ap.add_argument("--x-dtype", choices=["f32", "bf16"], default="f32",
                    help="activation type for --workload shape:M,K,N")
    ap.add_argument("--force-path", type=int, default=0, choices=[0, 1, 2, 3, 4],
                    help="shape workload: 0 auto, 1 CUDA-core GEMV, 2 tile GEMM, 3 stream-K tcgen05, "
                         "4 cluster GEMV")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch every call only after the previous one has finished")
    ap.add_argument("--tp-layers", type=int, default=48, help="tp_decode: layers of the GPT-2-XL-shaped model")
    ap.add_argument("--multi", choices=["sharded", "replicas"], default="sharded",
                    help="N > 1: the decode set column-sharded over the ranks (strong scaling, default) or "
                         "one full set per rank (replicas)")
    ap.add_argument("--exchange", choices=["fused", "separate"], default="fused",
                    help="N > 1, sharded decode set: the all-gather fused into the grouped GEMV (default) or run "
                         "after it (mtrtq_shard_allgather)")
    ap.add_argument("--step-launch", choices=["group", "hybrid", "calls"], default="group",
                    help="decode set: one grouped launch per step (default); hybrid: the eight smaller "
                         "calls grouped and the two LM heads as their own launches; calls: a launch per call")
    ap.add_argument("--branches", type=int, default=1,
                    help="decode set: run the step's independent calls as this many parallel graph branches")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, None, "fallback"


# Kernel (function name) that each plan path launches.
PATH_KERNELS = {"gemv": "gemv_q8_kernel", "gemm_tc": "gemm_q8_tc_kernel", "gemv_stream": "gemv_stream_kernel",
                "stream_k_tc": "skinny_q8_tc_kernel", "cluster_gemv": "gemv_cluster_kernel",
                "gemv_tc": "gemv_tc_kernel"}

# Arithmetic of each path: what the product is computed in.
PATH_DTYPES = {"gemv": "int8 W -> fp32, fp32 FMA",
               "gemv_stream": "int8 W x int8 activation digits (3 per value), int32 accumulate",
               "gemm_tc": "int8 W -> bf16, bf16 x bf16 tcgen05, fp32 accumulate",
               "stream_k_tc": "int8 W -> bf16, bf16 x bf16 tcgen05, fp32 accumulate",
               "cluster_gemv": "int8 W x int8 activation digits (3 per value), int32 accumulate",
               "gemv_tc": "int8 W x int8 activation digits (4 per value) on tcgen05 kind::i8, int32 accumulate"}


def committed_traffic(kernel_key: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(kernel_key)


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- ours


def build_decode_set(torch, dev, mode):
    from mini_tensorrt_b200 import matmulq, workloads as wl
    calls = []  # one entry per (M, shape): inputs, outputs, weight copies, workspace
    for M in wl.DECODE_M:
        for name, K, N in wl.DECODE_SHAPES:
            W = wl.decode_weight(name, K, N)
            q, s = matmulq.quantize_per_channel(W)
            base = matmulq.PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), dev)
            copies = [base] + [matmulq.PackedWeight(base.packed.clone(), base.scale.clone(), K, N)
                               for _ in range(WEIGHT_COPIES - 1)]
            x = torch.from_numpy(wl.activations(M, K, wl.shape_seed("x:" + name, M, K))).to(dev)
            y = torch.empty((M, N), dtype=torch.float32, device=dev)
            ws_bytes = matmulq.workspace_bytes(M, K, N, torch.float32, mode)
            ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
            calls.append({"name": name, "M": M, "K": K, "N": N, "x": x, "y": y, "w": copies,
                          "ws": ws, "bytes": wl.algorithmic_bytes(M, K, N, 4)})
    return calls


def branch_plan(calls, n_branches):
    """The step's calls on n_branches streams: the calls are independent, so the
    graph of a step forks into branches that the GPU runs side by side. Largest
    calls first, each to the branch with the fewest bytes so far."""
    loads = [0] * n_branches
    plan = [[] for _ in range(n_branches)]
    for i in sorted(range(len(calls)), key=lambda i: -calls[i]["bytes"]):
        b = loads.index(min(loads))
        plan[b].append(i)
        loads[b] += calls[i]["bytes"]
    return [p for p in plan if p]


def launch_step(calls, step, mode, stream, branches=None, side_streams=()):
    """One step: every call once, weights of copy (step + i) % WEIGHT_COPIES. With
    branches (lists of call indices), branch b > 0 runs on side_streams[b - 1],
    forked from and joined back into `stream` with events (inside a capture this
    makes parallel graph branches)."""
    import torch
    from mini_tensorrt_b200 import matmulq

    def one(i, st):
        c = calls[i]
        w = c["w"][(step + i) % WEIGHT_COPIES]
        matmulq.matmul_q8(c["x"], w, out=c["y"], mode=mode, workspace=c["ws"], stream=st)

    if not branches or len(branches) == 1:
        for i in range(len(calls)):
            one(i, stream)
        return
    fork = torch.cuda.Event()
    fork.record(stream)
    for b, idx in enumerate(branches):
        st = stream if b == 0 else side_streams[b - 1]
        if b > 0:
            st.wait_event(fork)
        for i in idx:
            one(i, st)
    for st in side_streams[:len(branches) - 1]:
        done = torch.cuda.Event()
        done.record(st)
        stream.wait_event(done)


def time_graphs(torch, graphs, steps, warmup, stream):
    """Replays graphs round-robin on `stream` (the timed replays continue the
    warm-up's order); returns seconds for `steps` replays."""
    with torch.cuda.stream(stream):
        for i in range(warmup):
            graphs[i % len(graphs)].replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(warmup, warmup + steps):
            graphs[i % len(graphs)].replay()
        e1.record(stream)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3


def time_step_graphs(torch, singles, pairs, steps, warmup, stream):
    """Like time_graphs over the rotation, but every two consecutive steps that start
    at an even rotation offset replay as one graph holding both (pairs[g // 2] is
    steps g and g + 1); a step left over replays alone. Every step still runs its
    full launch sequence on its own weight copy."""
    n = len(singles)

    def run(i0, count):
        i = i0
        while i < i0 + count:
            if i % 2 == 0 and i + 1 < i0 + count:
                pairs[(i % n) // 2].replay()
                i += 2
            else:
                singles[i % n].replay()
                i += 1

    with torch.cuda.stream(stream):
        run(0, warmup)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run(warmup, steps)
        e1.record(stream)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3


def run_ours(args, torch, rank, world, dev, dist):
    from mini_tensorrt_b200 import _lib, matmulq, workloads as wl
    hbm_peak, tc_peak, tc_sust, peak_kind = peaks()
    stream = torch.cuda.Stream(dev)
    # The decode set's weights are resident and never written inside the step, so
    # each call may start while the one ahead finishes (MTRTQ_OPT_OVERLAP_LAUNCH).
    matmulq.set_option(_lib.OPT_OVERLAP_LAUNCH, 0 if args.no_overlap else 1)
    calls = build_decode_set(torch, dev, args.mode)
    step_bytes = sum(c["bytes"] for c in calls)
    branches = branch_plan(calls, args.branches)
    side = [torch.cuda.Stream(dev) for _ in range(len(branches) - 1)]

    def capture_calls():
        """One graph per weight-copy rotation offset, a MatMulQ launch per call."""
        out = []
        with torch.cuda.stream(stream):
            launch_step(calls, 0, args.mode, stream, branches, side)  # first launch outside capture
            torch.cuda.synchronize()
            for g in range(WEIGHT_COPIES):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    launch_step(calls, g, args.mode, stream, branches, side)
                out.append(graph)
        torch.cuda.synchronize()
        return out

    # hybrid: the calls the grouped launch takes (all, or all but the LM heads, which
    # then run as their own cluster GEMV launches on the same stream).
    in_group = [i for i, c in enumerate(calls) if args.step_launch == "group" or c["name"] != "lm_head"]
    alone = [i for i in range(len(calls)) if i not in in_group]

    def capture_group():
        """One graph per rotation offset: the grouped launch (+ the LM heads alone)."""
        groups = [matmulq.GemvGroup([{"x": calls[i]["x"], "w": calls[i]["w"][(g + i) % WEIGHT_COPIES],
                                      "out": calls[i]["y"]} for i in in_group], mode=args.mode)
                  for g in range(WEIGHT_COPIES)]

        def one(g):
            groups[g](stream)
            for i in alone:
                c = calls[i]
                matmulq.matmul_q8(c["x"], c["w"][(g + i) % WEIGHT_COPIES], out=c["y"], mode=args.mode,
                                  workspace=c["ws"], stream=stream)
        out, pairs = [], []
        with torch.cuda.stream(stream):
            one(0)
            torch.cuda.synchronize()
            for g in range(WEIGHT_COPIES):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    one(g)
                out.append(graph)
            # two consecutive steps per graph: inside a graph the second step's
            # launches overlap the first's tail (programmatic dependent launch);
            # between graph replays they cannot
            for g in range(0, WEIGHT_COPIES, 2):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    one(g)
                    one(g + 1)
                pairs.append(graph)
        torch.cuda.synchronize()
        return out, groups, pairs

    groups, pairs = None, None
    if args.step_launch in ("group", "hybrid"):
        graphs, groups, pairs = capture_group()
    else:
        graphs = capture_calls()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        if world > 1:
            dist.barrier()
        if pairs is not None:
            secs = time_step_graphs(torch, graphs, pairs, args.steps, args.warmup, stream)
        else:
            secs = time_graphs(torch, graphs, args.steps, args.warmup, stream)
        if world > 1:
            dist.barrier()
    single_step = None
    if pairs is not None:
        s1 = time_graphs(torch, graphs, args.steps, args.warmup, stream)
        single_step = {"value": round(step_bytes * args.steps * world / s1 / 1e9, 1),
                       "ms_per_step": round(s1 / args.steps * 1e3, 4)}
    torch.cuda.synchronize()
    t = torch.tensor([secs], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs = float(t.item())
    value = step_bytes * args.steps * world / secs / 1e9
    assert matmulq.read_device_status() == 0, "a device wait timed out"
    step_us = secs / args.steps * 1e6
    other = None
    if args.step_launch != "calls":
        # The same step as ten MatMulQ launches (the cluster GEMV), for comparison.
        call_graphs = capture_calls()
        s2 = time_graphs(torch, call_graphs, args.steps, args.warmup, stream)
        other = {"step_launch": "calls", "value": round(step_bytes * args.steps / s2 / 1e9, 1),
                 "ms_per_step": round(s2 / args.steps * 1e3, 4)}
        del call_graphs

    # Dominant kernel: the LM head GEMVs (most of the bytes). Each is timed as it
    # runs in the step, back to back on the launching stream: one graph of
    # LAUNCHES_PER_GRAPH launches rotating over the weight copies (so every launch
    # reads its weights from HBM), CUDA events around the replays.
    per_kernel = {}
    for c in calls:
        if c["name"] != "lm_head":
            continue
        with torch.cuda.stream(stream):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for g in range(LAUNCHES_PER_GRAPH):
                    matmulq.matmul_q8(c["x"], c["w"][g % WEIGHT_COPIES], out=c["y"],
                                      mode=args.mode, workspace=c["ws"], stream=stream)
        reps = max(10, args.steps // 2)
        s = time_graphs(torch, [graph], reps, 3, stream)
        per_kernel[c["M"]] = {"us": s / (reps * LAUNCHES_PER_GRAPH) * 1e6, "bytes": c["bytes"],
                              "plan": matmulq.plan_info(c["M"], c["K"], c["N"], mode=args.mode)}
        del graph
    # the LM head launch with the larger time is the dominant kernel of the per-call step
    dom_m = max(per_kernel, key=lambda m: per_kernel[m]["us"])
    dom = per_kernel[dom_m]
    lm_achieved = dom["bytes"] / (dom["us"] * 1e-6) / 1e9
    lm_head = {"kernel": f"{PATH_KERNELS[dom['plan']['path']]} (LM head 768x50257, M={dom_m})",
               "achieved": round(lm_achieved, 1), "frac": round(lm_achieved / hbm_peak, 4),
               "per_launch_us": round(dom["us"], 3), "algorithmic_bytes_per_launch": dom["bytes"],
               "traffic": committed_traffic(f"gemv_lm_head_m{dom_m}_{args.mode}"),
               "other_m": {str(m): round(v["us"], 3) for m, v in per_kernel.items()}}
    if args.step_launch == "group":
        # One grouped GEMV per step (with its digitize launch ahead of it, the two
        # overlapped by programmatic dependent launch): the step time measured
        # above bounds the GEMV's launch duration from above, so the fraction is
        # a lower bound.
        achieved = step_bytes / (step_us * 1e-6) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(achieved / hbm_peak, 4),
                    "traffic": committed_traffic(f"gemv_tc_decode_set_{args.mode}"),
                    "kernel": "gemv_tc_kernel (the whole decode GEMV set, one launch, after its digitize_kernel)",
                    "peak_kind": f"{peak_kind} hbm_gbs", "per_launch_us": round(step_us, 3),
                    "per_launch_timing": "CUDA events around graph replays of two steps each (digitize + grouped "
                                         f"GEMV per step), weights rotated over {WEIGHT_COPIES} copies",
                    "algorithmic_bytes_per_launch": step_bytes,
                    "lm_head_per_call": lm_head}
    else:
        roofline = {"bound": "hbm", "achieved": lm_head["achieved"], "peak": hbm_peak, "unit": "GB/s",
                    "frac": lm_head["frac"], "traffic": lm_head["traffic"], "kernel": lm_head["kernel"],
                    "peak_kind": f"{peak_kind} hbm_gbs", "per_launch_us": lm_head["per_launch_us"],
                    "per_launch_timing": f"mean over graphs of {LAUNCHES_PER_GRAPH} back-to-back "
                                         f"launches, weights rotated over {WEIGHT_COPIES} copies",
                    "algorithmic_bytes_per_launch": dom["bytes"]}

    # End to end through the C ABI from the host (pinned buffers, copies timed).
    e2e = run_e2e(torch, calls, args, dev, stream, dist, world)
    if args.step_launch == "group":
        per_call = e2e
        e2e = run_e2e_group(torch, calls, args, dev, stream, dist, world)
        e2e["per_call_c_abi"] = per_call

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": PATH_DTYPES["gemv_tc" if args.step_launch == "group" else "cluster_gemv"],
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights quantized per channel)",
        "config": decode_set_config(args, world, step_bytes),
        "method": {"timing": ("CUDA graphs of two consecutive steps (a step left over alone), CUDA events on "
                              "the launching stream" if pairs is not None else
                              "CUDA graphs of one step, CUDA events on the launching stream"),
                   "one_step_per_graph": single_step,
                   "overlap_launch": not args.no_overlap,
                   "step_launch": {"group": "one mtrtq_gemv_group call for the ten calls (a digitize kernel and "
                                             "the tensor-core digit GEMV)",
                                   "hybrid": "one mtrtq_gemv_group launch for the eight smaller calls, then the two "
                                             "LM heads as cluster GEMV launches",
                                   "calls": "one MatMulQ launch per call"}[args.step_launch],
                   "graph_branches": (None if args.step_launch != "calls" else
                                      [[calls[i]["name"] + f"/M{calls[i]['M']}" for i in b] for b in branches]),
                   "other_step_launch": other},
        "roofline": roofline,
        "e2e": e2e,
        # group: the digitize kernel and the grouped GEMV; hybrid: those and the two
        # LM heads; calls: one kernel per call.
        "gpu_launches": {"group": 2, "hybrid": 2 + len(alone), "calls": len(calls)}[args.step_launch] * args.steps,
        "clocks": clk.summary(),
    }
    return line, calls, stream


def run_sharded_decode_set(args, torch, rank, world, dev, dist):
    """The decode GEMV set strong-scaled over the ranks: every call's output
    channels split into whole 128-channel tiles per rank (mtrtq_shard_range), a
    step = one grouped launch of this rank's shards writing straight into its copy
    of the outputs, then one all-gather of every rank's output segments through
    peer memory (mtrtq_shard_allgather), so that every rank ends the step with all
    ten full outputs. Both launches are captured in one CUDA graph per weight
    rotation (the exchange counts its epochs on the device). value = the unsplit
    step's algorithmic bytes x steps / the max over ranks of the timed region."""
    from mini_tensorrt_b200 import _lib, matmulq, sharded, workloads as wl
    hbm_peak, _, _, peak_kind = peaks()
    matmulq.set_option(_lib.OPT_OVERLAP_LAUNCH, 0 if args.no_overlap else 1)
    shapes = [(M, name, K, N) for M in wl.DECODE_M for name, K, N in wl.DECODE_SHAPES]
    y_elems = sum(M * N for M, _, _, N in shapes)
    # outputs alternate between two copies from one step to the next (graph g
    # writes copy g % 2; the rotation count is even), so no entry barrier is needed
    peers = sharded.PeerBuffers(y_elems, 0, device=dev, device_epochs=True, alternating=True)
    assert WEIGHT_COPIES % 2 == 0
    calls, off, step_bytes, my_bytes = [], 0, 0, 0
    for M, name, K, N in shapes:
        n0, n1 = sharded.shard_range(N, "N", rank, world)
        c = {"name": name, "M": M, "K": K, "N": N, "n0": n0, "n1": n1, "off": off,
             "x": torch.from_numpy(wl.activations(M, K, wl.shape_seed("x:" + name, M, K))).to(dev)}
        step_bytes += wl.algorithmic_bytes(M, K, N, 4)
        if n1 > n0:
            q, s = matmulq.quantize_per_channel(wl.decode_weight(name, K, N))
            base = matmulq.PackedWeight.from_int8(torch.from_numpy(np.ascontiguousarray(q[:, n0:n1])),
                                                  torch.from_numpy(np.ascontiguousarray(s[n0:n1])), dev)
            c["w"] = [base] + [matmulq.PackedWeight(base.packed.clone(), base.scale.clone(), K, n1 - n0)
                               for _ in range(WEIGHT_COPIES - 1)]
            my_bytes += K * (n1 - n0)
        calls.append(c)
        off += M * N
    mine = [c for c in calls if c["n1"] > c["n0"]]

    def out_view(c, g):
        o = (g % 2) * y_elems + c["off"]
        return peers.y[o:o + c["M"] * c["N"]].view(c["M"], c["N"])

    segments = [[((g % 2) * y_elems + c["off"] + c["n0"], c["M"], c["n1"] - c["n0"], c["N"]) for c in mine]
                for g in range(2)]
    groups = [matmulq.GemvGroup([{"x": c["x"], "w": c["w"][(g + i) % WEIGHT_COPIES],
                                  "out": out_view(c, g)[:, c["n0"]:c["n1"]]} for i, c in enumerate(mine)],
                                mode=args.mode)
              for g in range(WEIGHT_COPIES)]
    stream = torch.cuda.Stream(dev)

    def one(g):
        if args.exchange == "fused":  # one call: the group's kernel stores to every rank
            peers.group_allgather(groups[g], stream=stream)
        else:
            groups[g](stream)
            peers.allgather(segments[g % 2], stream=stream)

    graphs = []
    with torch.cuda.stream(stream):
        one(0)  # eager set-up launches, copy 0 then copy 1, so that the replays
        one(1)  # (graph 0 first) keep alternating
        torch.cuda.synchronize()
        for g in range(WEIGHT_COPIES):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                one(g)
            graphs.append(graph)
    torch.cuda.synchronize()
    dist.barrier()
    with ClockSampler(dev.index) as clk:
        dist.barrier()
        secs = time_graphs(torch, graphs, args.steps, args.warmup, stream)
        dist.barrier()
    t = torch.tensor([secs], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs = float(t.item())
    assert matmulq.read_device_status() == 0, "a device wait timed out"
    # every rank holds the full outputs: check them against this rank's own
    # unsplit product of the last step's weights (sampled rows of each call)
    last = (args.steps + args.warmup - 1) % WEIGHT_COPIES  # the graph of the last step
    for c in calls:
        full_q, full_s = matmulq.quantize_per_channel(wl.decode_weight(c["name"], c["K"], c["N"]))
        pw = matmulq.PackedWeight.from_int8(torch.from_numpy(full_q), torch.from_numpy(full_s), dev)
        ref = matmulq.matmul_q8(c["x"], pw, mode=args.mode)
        torch.cuda.synchronize()
        err = float((out_view(c, last) - ref).abs().max() / ref.abs().max())
        assert err <= 1e-4, f"sharded step output {c['name']}/M{c['M']} differs from the unsplit product: {err:.3e}"
    step_us = secs / args.steps * 1e6
    exch_bytes = sum(c["M"] * c["N"] * 4 for c in calls) * (world - 1) / world  # each rank receives
    line = {"value": round(step_bytes * args.steps / secs / 1e9, 1), "ms_per_step": round(step_us / 1e3, 4),
            "scaling": "strong", "clocks": clk.summary(),
            "rank0_weight_bytes_per_step": my_bytes,
            "exchange": {"how": ("mtrtq_gemv_group_allgather: the grouped GEMV's epilogue stores every output to "
                                 "every rank over NVLink; its last CTA signals the peers and waits, bounded, for "
                                 "theirs (one call per step)") if args.exchange == "fused" else
                                ("mtrtq_shard_allgather after the group: peer stores, bounded wait (library "
                                 "kernels)"),
                         "bytes_received_per_rank_per_step": int(exch_bytes),
                         "nvlink_lower_bound_us": round(exch_bytes / 770e9 * 1e6, 3)},
            # per step: the digitize kernel and the grouped GEMV (fused: it also
            # stores to the peers), or those, then the all-gather's epoch kernel
            # (device-counted epochs) and push kernel
            "gpu_launches": (2 if args.exchange == "fused" else 4) * args.steps}
    del graphs
    peers.close()
    return line


def run_e2e_group(torch, calls, args, dev, stream, dist, world):
    """End to end through the grouped API with host buffers: per step, one pinned
    H2D copy of the ten calls' activations (packed in one buffer), one
    mtrtq_gemv_group launch, one pinned D2H copy of the ten outputs. Steps alternate
    between two streams, each with its own device buffers, so one step's copies
    overlap the other's launch; the timed region ends when both streams have
    delivered their last outputs."""
    from mini_tensorrt_b200 import matmulq
    xs = sum(c["M"] * c["K"] for c in calls)
    ys = sum(c["M"] * c["N"] for c in calls)
    hx = torch.cat([c["x"].reshape(-1).cpu() for c in calls]).pin_memory()
    step_bytes = sum(c["bytes"] for c in calls)
    sets = []
    for b in range(2):
        st = stream if b == 0 else torch.cuda.Stream(dev)
        dx = torch.empty(xs, device=dev)
        dy = torch.empty(ys, device=dev)
        hy = torch.empty(ys).pin_memory()
        views, ox, oy = [], 0, 0
        for c in calls:
            views.append((dx[ox:ox + c["M"] * c["K"]].view(c["M"], c["K"]),
                          dy[oy:oy + c["M"] * c["N"]].view(c["M"], c["N"])))
            ox += c["M"] * c["K"]
            oy += c["M"] * c["N"]
        groups = [matmulq.GemvGroup([{"x": views[i][0], "w": c["w"][(g + i) % WEIGHT_COPIES], "out": views[i][1]}
                                     for i, c in enumerate(calls)], mode=args.mode) for g in range(WEIGHT_COPIES)]
        sets.append((st, dx, dy, hy, groups))

    def step(i):
        st, dx, dy, hy, groups = sets[i % 2]
        with torch.cuda.stream(st):
            dx.copy_(hx, non_blocking=True)
            groups[i % WEIGHT_COPIES](st)
            hy.copy_(dy, non_blocking=True)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    sets[1][0].wait_event(e0)
    for i in range(args.steps):
        step(i)
    done = torch.cuda.Event()
    done.record(sets[1][0])
    stream.wait_event(done)
    e1.record(stream)
    torch.cuda.synchronize()
    # the outputs of the last step delivered to the host are the device's
    last = sets[(args.steps - 1) % 2]
    assert torch.equal(last[3], last[2].cpu())
    secs = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([secs], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs = float(t.item())
    return {"value": round(step_bytes * args.steps * world / secs / 1e9, 1), "unit": UNIT,
            "h2d_bytes_per_step": xs * 4, "d2h_bytes_per_step": ys * 4,
            "ms_per_step": round(secs / args.steps * 1e3, 4),
            "how": "per step: one pinned H2D of the ten X (packed), one mtrtq_gemv_group launch, one pinned D2H "
                   "of the ten Y; steps alternate over two streams with their own device buffers; CUDA events "
                   "around the steps"}


def run_e2e(torch, calls, args, dev, stream, dist, world):
    """The reference-facing call with host buffers: per call, mtrtq_matmul_host (one
    C-ABI call: pinned H2D of X, the product, D2H of Y, enqueued on one stream).
    The step's calls are independent, so they go round-robin over E2E_STREAMS
    streams (each call keeps its stream and workspace across steps): one call's
    copies overlap another's kernel. The timed region ends when every stream has
    delivered its last result."""
    from mini_tensorrt_b200 import _lib, matmulq
    from mini_tensorrt_b200.matmulq import MODES
    lib = _lib.lib()
    hx = [c["x"].cpu().pin_memory() for c in calls]
    hy = [torch.empty_like(c["y"], device="cpu").pin_memory() for c in calls]
    streams = [stream] + [torch.cuda.Stream(dev) for _ in range(E2E_STREAMS - 1)]
    mode = MODES[args.mode]
    h2d = sum(c["M"] * c["K"] * 4 for c in calls)
    d2h = sum(c["M"] * c["N"] * 4 for c in calls)
    step_bytes = sum(c["bytes"] for c in calls)
    wss = [torch.zeros(matmulq.host_workspace_bytes(c["M"], c["K"], c["N"], args.mode),
                       dtype=torch.uint8, device=dev) for c in calls]
    ptrs = [(hx[j].data_ptr(), hy[j].data_ptr(), c["M"], c["K"], c["N"], wss[j].data_ptr(),
             wss[j].numel(), [w.packed.data_ptr() for w in c["w"]], [w.scale.data_ptr() for w in c["w"]],
             streams[j % E2E_STREAMS].cuda_stream)
            for j, c in enumerate(calls)]
    fn = lib.mtrtq_matmul_host

    def step(i):
        for j, (xp, yp, M, K, N, wsp, wsn, wps, sps, sp) in enumerate(ptrs):
            g = (i + j) % WEIGHT_COPIES
            rc = fn(xp, wps[g], sps[g], None, yp, M, K, N, mode, wsp, wsn, 0, sp)
            if rc != 0:
                raise RuntimeError(_lib.last_error())

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in streams[1:]:
        s.wait_event(e0)
    for i in range(args.steps):
        step(i)
    for s in streams[1:]:
        done = torch.cuda.Event()
        done.record(s)
        stream.wait_event(done)
    e1.record(stream)
    torch.cuda.synchronize()
    secs = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([secs], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs = float(t.item())
    return {"value": round(step_bytes * args.steps * world / secs / 1e9, 1), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(secs / args.steps * 1e3, 4),
            "how": f"per call: mtrtq_matmul_host via ctypes (pinned H2D of X, product, pinned "
                   f"D2H of Y on one stream), the step's independent calls round-robin over "
                   f"{E2E_STREAMS} streams; CUDA events around the steps"}


def run_extras(torch, dev, args, stream):
    """Prefill tensor-core GEMM at the large shapes (M=2048, bf16 X) and the
    single-op FFN-up case (M=64, fp32 X, bias), each timed alone."""
    from mini_tensorrt_b200 import matmulq, workloads as wl
    hbm_peak, tc_peak, tc_sust, peak_kind = peaks()
    out = {}
    for (K, N) in wl.LARGE_SHAPES:
        M = 2048
        W = wl.weights(K, N, wl.shape_seed(f"large_{K}x{N}", K, N))
        q, s = matmulq.quantize_per_channel(W)
        pw = matmulq.PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), dev)
        x = torch.randn(M, K, device=dev, generator=torch.Generator(dev).manual_seed(1)).to(torch.bfloat16)
        y = torch.empty(M, N, device=dev)
        ws = torch.zeros(max(matmulq.workspace_bytes(M, K, N, torch.bfloat16, "bf16"), 256),
                         dtype=torch.uint8, device=dev)
        with torch.cuda.stream(stream):
            matmulq.matmul_q8(x, pw, out=y, workspace=ws, stream=stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(5):
                    matmulq.matmul_q8(x, pw, out=y, workspace=ws, stream=stream)
        secs = time_graphs(torch, [graph], 10, 3, stream) / 5
        tf = wl.flops(M, K, N) / (secs / 10) / 1e12
        out[f"gemm_m{M}_{K}x{N}"] = {"tflops": round(tf, 1), "us": round(secs / 10 * 1e6, 2),
                                     "frac_of_bf16_peak": round(tf / tc_peak, 4),
                                     "plan": matmulq.plan_info(M, K, N, torch.bfloat16, "bf16")}
        del pw, x, y, ws, graph
    M, K, N = 64, 768, 3072
    W = wl.weights(K, N, 7)
    q, s = matmulq.quantize_per_channel(W)
    copies = [matmulq.PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), dev)
              for _ in range(60)]  # 141 MB of weights > L2
    x = torch.randn(M, K, device=dev)
    b = torch.randn(N, device=dev) * 0.02
    y = torch.empty(M, N, device=dev)
    byts = wl.algorithmic_bytes(M, K, N, 4, True)
    for mode in ("fp32", "bf16"):
        ws = torch.zeros(max(matmulq.workspace_bytes(M, K, N, torch.float32, mode), 256),
                         dtype=torch.uint8, device=dev)
        with torch.cuda.stream(stream):
            matmulq.matmul_q8(x, copies[0], bias=b, out=y, mode=mode, workspace=ws, stream=stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for c in copies:
                    matmulq.matmul_q8(x, c, bias=b, out=y, mode=mode, workspace=ws, stream=stream)
        secs = time_graphs(torch, [graph], 5, 2, stream) / (5 * len(copies))
        key = "single_op_ffn_up_m64_bias" + ("" if mode == "fp32" else "_bf16")
        out[key] = {"mode": mode, "us": round(secs * 1e6, 2), "gbs": round(byts / secs / 1e9, 1),
                    "hbm_frac": round(byts / secs / 1e9 / hbm_peak, 4),
                    "tflops": round(wl.flops(M, K, N) / secs / 1e12, 2),
                    "plan": matmulq.plan_info(M, K, N, torch.float32, mode),
                    "timing": f"one graph of {len(copies)} back-to-back calls over distinct weight copies"}
        del graph
    return out


def run_shape(args, torch, dev):
    """One MatMulQ shape timed alone: one CUDA graph of back-to-back launches over
    enough weight copies to exceed 2x L2, replayed --steps times."""
    from mini_tensorrt_b200 import matmulq, workloads as wl
    hbm_peak, tc_peak, _, peak_kind = peaks()
    M, K, N = (int(v) for v in args.workload.split(":", 1)[1].split(","))
    matmulq.set_option(2, args.force_path)  # MTRTQ_OPT_FORCE_PATH
    W = wl.weights(K, N, wl.shape_seed("shape", K, N))
    q, s = matmulq.quantize_per_channel(W)
    base = matmulq.PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), dev)
    n_copies = max(2, -(-(260 << 20) // (K * N)))
    copies = [base] + [matmulq.PackedWeight(base.packed.clone(), base.scale, K, N)
                       for _ in range(n_copies - 1)]
    xdt = torch.bfloat16 if args.x_dtype == "bf16" else torch.float32
    x = torch.randn(M, K, device=dev, generator=torch.Generator(dev).manual_seed(1)).to(xdt)
    y = torch.empty(M, N, device=dev)
    ws = torch.zeros(max(matmulq.workspace_bytes(M, K, N, xdt, args.mode), 256), dtype=torch.uint8,
                     device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        matmulq.matmul_q8(x, copies[0], out=y, mode=args.mode, workspace=ws, stream=stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()   # one launch per weight copy, back to back
        with torch.cuda.graph(graph, stream=stream):
            for cpy in copies:
                matmulq.matmul_q8(x, cpy, out=y, mode=args.mode, workspace=ws, stream=stream)
    secs = time_graphs(torch, [graph], args.steps, args.warmup, stream) / (args.steps * n_copies)
    byts = wl.algorithmic_bytes(M, K, N, 2 if xdt == torch.bfloat16 else 4)
    plan = matmulq.plan_info(M, K, N, xdt, args.mode)
    matmulq.set_option(2, 0)
    return {"workload": args.workload, "x_dtype": args.x_dtype, "mode": args.mode,
            "us_per_call": round(secs * 1e6, 3), "gbs": round(byts / secs / 1e9, 1),
            "hbm_frac": round(byts / secs / 1e9 / hbm_peak, 4),
            "tflops": round(wl.flops(M, K, N) / secs / 1e12, 2),
            "tc_frac": round(wl.flops(M, K, N) / secs / 1e12 / tc_peak, 4),
            "peak_kind": peak_kind, "weight_copies": n_copies, "plan": plan}


def run_gpt2_decode(args, torch, dev, mode=None):
    """Random-init GPT-2 small, every Linear an int8 MatMulQ, greedy KV-cache decoding
    on the device (one CUDA graph per step): prompts of 64 ids, then 64 generated
    tokens, batch 1 and 16, the prompt prefilled token by token (as the reference
    does) and in one pass of M = B * 64 products. Reports prefill and decode
    tokens/s (all sequences) and the decode steps' weight bytes per second (int8
    Linears + tied LM head). The default mode is fp32, whose tokens are identical to
    the reference decoder's at both batches (bf16 mode flips a few near-tie
    argmaxes at batch 16)."""
    from mini_tensorrt_b200 import gpt2
    from mini_tensorrt_b200.matmulq import set_option
    from mini_tensorrt_b200 import _lib
    mode = mode or args.mode
    set_option(_lib.OPT_OVERLAP_LAUNCH, 0 if args.no_overlap else 1)
    cfg = gpt2.GPT2Config()
    w = gpt2.random_weights(cfg, seed=0)
    P, new = 64, 64
    D, F, V, L = cfg.d_model, cfg.d_ff, cfg.vocab, cfg.n_layer
    step_bytes = L * (D * 3 * D + D * D + D * F + F * D) + D * V
    out = {"workload": "gpt2_decode",
           "config": {"model": "GPT-2 small (12L, d 768, 12 heads, d_ff 3072, vocab 50257), random init",
                      "prompt_len": P, "max_new": new, "mode": mode,
                      "weight_bytes_per_step": step_bytes,
                      "timing": "CUDA events around the prefill and around the graph replays of the decode steps"},
           "batches": {}}
    for B in (1, 16):
        dec = gpt2.DeviceDecoder(w, B, max_ctx=P + new, mode=mode, device=dev)
        prompt = np.random.default_rng(1234 + B).integers(0, V, (B, P), dtype=np.int32)
        row = {}
        for pf in ("tokens", "gemm"):
            dec.generate(prompt, new, prefill=pf)  # capture + warm-up
            runs = [dec.generate(prompt, new, prefill=pf) for _ in range(3)]
            dsec = min(r["decode_s"] for r in runs)
            psec = min(r["prefill_s"] for r in runs)
            nsteps = new - 1
            row["decode_tok_s"] = round(B * nsteps / dsec, 1)
            row["decode_ms_per_step"] = round(dsec / nsteps * 1e3, 4)
            row["decode_weight_gbs"] = round(step_bytes * nsteps / dsec / 1e9, 1)
            row[f"prefill_{pf}_tok_s"] = round(B * P / psec, 1)
            row[f"prefill_{pf}_ms"] = round(psec * 1e3, 3)
        out["batches"][str(B)] = row
        del dec
        torch.cuda.empty_cache()
    return out


def run_tp_decode(args, torch, rank, world, dev, dist):
    """GPT-2-XL-shaped random-init model (48 layers, d 1600, 25 heads, d_ff 6400,
    vocab 50257), every Linear int8 per channel, tensor-parallel over the ranks
    (mini_tensorrt_b200.tp: column-split QKV by heads and FFN-up, row-split
    attn-out and FFN-down with two library all-reduces per layer, vocabulary-split
    LM head): batch 32, prompts of 128 ids consumed token by token, then 128 greedy
    tokens; one CUDA graph per step on every rank. Reports decode tokens/s over all
    sequences (max over ranks of the decode time) and checks that every rank
    produced the same tokens. --tp-layers shortens the model for quick runs."""
    import dataclasses
    from mini_tensorrt_b200 import gpt2, tp
    from mini_tensorrt_b200.matmulq import set_option
    from mini_tensorrt_b200 import _lib
    set_option(_lib.OPT_OVERLAP_LAUNCH, 0 if args.no_overlap else 1)
    cfg = dataclasses.replace(tp.GPT2_XL, n_layer=args.tp_layers)
    B, P, new = 32, 128, 128
    t0 = time.time()
    w = gpt2.random_weights(cfg, seed=0)
    setup_s = time.time() - t0
    dec = tp.TPDecoder(w, B, max_ctx=P + new, mode=args.mode, device=dev)
    del w
    prompt = np.random.default_rng(4321).integers(0, cfg.vocab, (B, P), dtype=np.int32)
    dec.generate(prompt, 8)  # capture + warm-up
    runs = []
    for _ in range(2):
        if world > 1:
            dist.barrier()
        runs.append(dec.generate(prompt, new))
    dsec = min(r["decode_s"] for r in runs)
    t = torch.tensor([dsec], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dsec = float(t.item())
    toks = torch.from_numpy(runs[-1]["tokens"]).to(dev)
    if world > 1:
        allt = [torch.empty_like(toks) for _ in range(world)]
        dist.all_gather(allt, toks)
        assert all(torch.equal(allt[0], a) for a in allt), "ranks generated different tokens"
    D, F, V, L = cfg.d_model, cfg.d_ff, cfg.vocab, cfg.n_layer
    step_bytes = L * (D * 3 * D + D * D + D * F + F * D) + D * V
    nsteps = new - 1
    digest = int(np.asarray(runs[-1]["tokens"], dtype=np.int64).sum())
    dec.close()
    return {"metric": METRIC, "impl": "ours", "workload": "tp_decode", "n_gpus": world, "scaling": "strong",
            "config": {"model": f"GPT-2-XL shape ({L}L, d 1600, 25 heads, d_ff 6400, vocab 50257), random init",
                       "batch": B, "prompt_len": P, "max_new": new, "mode": args.mode,
                       "parallelism": f"tensor parallel x{world} (heads / FFN columns / vocabulary)",
                       "int8_weight_bytes_per_step": step_bytes},
            "decode_tok_s": round(B * nsteps / dsec, 1), "decode_ms_per_step": round(dsec / nsteps * 1e3, 4),
            "decode_weight_gbs": round(step_bytes * nsteps / dsec / 1e9, 1),
            "weight_bytes_per_rank_per_step": int(step_bytes / world),
            "exchanges_per_step": 2 * L + 1, "token_digest": digest, "weights_setup_s": round(setup_s, 1),
            "timing": "CUDA events around the 127 decode steps (graph replays), best of 2, max over ranks"}


def run_sharded(args, torch, rank, world, dev, dist):
    """One large MatMulQ split across the ranks (strong scaling: the total work is
    fixed): --workload sharded:M,K,N,S with S = N (column split + all-gather) or
    K (row split + all-reduce). Each rank rotates through copies of its shard
    (> 2x L2 per GPU); a call is the local product plus the collective, timed with
    CUDA events on the rank's stream, max over ranks. Also times the local product
    alone, and gives the collective's NVLink lower bound (770 GB/s per direction)."""
    from mini_tensorrt_b200 import matmulq, sharded, workloads as wl
    hbm_peak, tc_peak, _, peak_kind = peaks()
    M, K, N, split = args.workload.split(":", 1)[1].split(",")
    M, K, N = int(M), int(K), int(N)
    W = wl.weights(K, N, wl.shape_seed("sharded", K, N))
    q, s = matmulq.quantize_per_channel(W)
    op = sharded.ShardedMatMulQ(q, s, None, split=split, device=dev, mode=args.mode)
    b, e = op.shard.begin, op.shard.end
    shard_bytes = max(1, op.w.packed.numel())
    n_copies = max(2, -(-(260 << 20) // shard_bytes))
    copies = [op.w] + [matmulq.PackedWeight(op.w.packed.clone(), op.w.scale, op.w.K, op.w.N)
                       for _ in range(n_copies - 1)]
    xdt = torch.bfloat16 if args.x_dtype == "bf16" else torch.float32
    x = torch.randn(M, K, device=dev, generator=torch.Generator(dev).manual_seed(1)).to(xdt)

    def timed(fn, steps, warmup):
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3 / steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def full(i):
        op.w = copies[i % n_copies]
        op(x)

    xs = x[:, b:e] if split == "K" else x

    def local(i):
        matmulq.matmul_q8(xs, copies[i % n_copies], mode=args.mode)

    steps = max(args.steps, 2 * n_copies)
    t_call = timed(full, steps, max(args.warmup, n_copies))
    t_local = timed(local, steps, max(args.warmup, n_copies))
    out_bytes = M * N * 4
    if world == 1:
        comm_bytes = 0
    elif split == "N":
        comm_bytes = out_bytes * (world - 1) / world      # each GPU receives the other shards
    else:
        comm_bytes = 2 * out_bytes * (world - 1) / world  # ring all-reduce, per GPU
    byts = wl.algorithmic_bytes(M, K, N, 2 if xdt == torch.bfloat16 else 4)
    return {"metric": METRIC, "impl": "ours", "workload": args.workload, "n_gpus": world,
            "scaling": "strong", "split": split, "mode": args.mode, "x_dtype": args.x_dtype,
            "us_per_call": round(t_call * 1e6, 3), "us_local_product": round(t_local * 1e6, 3),
            "tflops": round(wl.flops(M, K, N) / t_call / 1e12, 2),
            "gbs": round(byts / t_call / 1e9, 1),
            "comm_lower_bound_us": round(comm_bytes / 770e9 * 1e6, 3),
            "shard": [b, e], "weight_copies_per_gpu": n_copies, "peak_kind": peak_kind,
            "timing": "CUDA events around eager calls (product + collective), max over ranks"}


# ---------------------------------------------------------------------- CPU legs


def _workloads():
    """mini_tensorrt_b200/workloads.py (seeded numpy inputs) loaded by file path,
    so the CPU legs import nothing else of the package: no libmtrtq.so, no torch."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "_mtrtq_workloads", os.path.join(ROOT, "mini_tensorrt_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def decode_set_calls():
    """The decode GEMV set's calls as the CPU legs see them: (name, X f32 [M,K],
    q int8 [K,N], scale f32 [N]); packed by the oracle's restatement of the
    reference packer (bit-exact with it)."""
    import oracle
    wl = _workloads()
    calls, step_bytes = [], 0
    packed = {}
    for M in wl.DECODE_M:
        for name, K, N in wl.DECODE_SHAPES:
            if name not in packed:
                packed[name] = oracle.quantize_per_channel(wl.decode_weight(name, K, N))
            q, s = packed[name]
            X = wl.activations(M, K, wl.shape_seed("x:" + name, M, K))
            calls.append((name, X, q, s))
            step_bytes += wl.algorithmic_bytes(M, K, N, 4)
    return calls, step_bytes


def decode_set_config(args, world, step_bytes):
    """The workload as both arms name it (identical dicts, so the two lines compare)."""
    return {"workload": DECODE_SET_WORKLOAD, "calls_per_step": 10, "algorithmic_bytes_per_step": step_bytes,
            "mode": args.mode, "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": f"inputs larger than L2: the GPU arm rotates every call over {WEIGHT_COPIES} device copies "
                  f"of its weights ({WEIGHT_COPIES * DECODE_SET_WEIGHT_BYTES / 1e6:.0f} MB > 2x the 126 MB L2); "
                  f"the CPU arm reads one host copy"}


def cpu_row_tasks(calls, chunk_cols=1000):
    """Independent pieces of the step for a pool of host threads: every call split
    by rows and by column chunks of <= chunk_cols. Rows and columns are
    independent in the reference loop (src/ops/kernels_matmul.cpp:66-73), and each
    piece runs the unmodified reference kernel on its own slice. The chunk width
    is the best measured for that kernel: its inner loop strides W by N bytes, and
    a power-of-two stride (4096) maps every k to the same cache sets; on one x86
    core an LM head row took 134 ms whole, 218 ms in 4096-column chunks and 51 ms
    in 1000-column chunks."""
    import oracle
    tasks = []
    for _, X, q, s in calls:
        N = q.shape[1]
        for r in range(X.shape[0]):
            for j0 in range(0, N, chunk_cols):
                j1 = min(N, j0 + chunk_cols)
                tasks.append(oracle.RefMatmulqCall(X[r:r + 1], np.ascontiguousarray(q[:, j0:j1]), s[j0:j1]))
    return tasks


def run_pool(tasks, threads, min_seconds=None, steps=None):
    """Runs whole steps of `tasks` (objects with run(), called from host threads;
    the C calls release the GIL) on `threads` threads; returns (steps, seconds)."""
    order = sorted(tasks, key=lambda t: -(t.M * t.N))  # longest first

    def run_step():
        if threads == 1:
            for t in order:
                t.run()
            return
        idx = [0]
        lock = threading.Lock()

        def worker():
            while True:
                with lock:
                    i = idx[0]
                    idx[0] += 1
                if i >= len(order):
                    return
                order[i].run()
        ws = [threading.Thread(target=worker) for _ in range(threads)]
        for w in ws:
            w.start()
        for w in ws:
            w.join()

    n, t0 = 0, time.perf_counter()
    while True:
        run_step()
        n += 1
        el = time.perf_counter() - t0
        if steps is not None and n >= steps:
            break
        if min_seconds is not None and el >= min_seconds:
            break
    return n, time.perf_counter() - t0


class _GemmAutoCall:
    """One call of the reference's fp32 gemm_auto (backends/cpu/gemm.cpp:288-302) on
    the dequantized weights q * scale: its own thread rule (the ThreadPool's
    hardware_concurrency() threads when M >= 32 and 2MNK >= 2^21, one otherwise)."""

    def __init__(self, X, q, s):
        import oracle
        self.X = np.ascontiguousarray(X, np.float32)
        self.W = np.ascontiguousarray(q.astype(np.float32) * s[None, :])
        self.M, self.N = X.shape[0], q.shape[1]
        self.C = np.zeros((self.M, self.N), np.float32)
        self._fn = oracle.ref().ref_gemm_auto
        self._args = (oracle._ptr(self.X, oracle._f32p), oracle._ptr(self.W, oracle._f32p),
                      oracle._ptr(self.C, oracle._f32p), self.M, self.N, self.X.shape[1])

    def run(self):
        self._fn(*self._args)


def cpu_baseline_line(calls, step_bytes, seconds=8.0):
    """The reference's CPU paths on this host, timed beside the GPU: (1) its MatMulQ
    kernel, single-threaded as it runs, each call prepared once and timed as the
    kernel call alone; (2) its fp32 'NEON / multithreaded' gemm_auto on dequantized
    weights with its own thread rule (on x86-64 its NEON step is the scalar packed
    fallback, gemm.cpp:251-254; at M < 32 it runs on one thread)."""
    import oracle
    if not oracle.ref_available():
        return {"value": None, "unit": UNIT, "cores": 1, "kind": "port",
                "sample": "oracle/_ref missing on this host"}
    mq = [oracle.RefMatmulqCall(X, q, s) for _, X, q, s in calls]
    n, secs = run_pool(mq, 1, min_seconds=seconds)
    mq_val = step_bytes * n / secs / 1e9
    ga = [_GemmAutoCall(X, q, s) for _, X, q, s in calls]
    n2, secs2 = run_pool(ga, 1, min_seconds=seconds)
    ga_val = step_bytes * n2 / secs2 / 1e9
    hw = int(oracle.ref().ref_hardware_threads())
    ga_threads = max(1 if X.shape[0] < 32 else hw for _, X, _, _ in calls)
    return {"value": round(mq_val, 4), "unit": UNIT, "cores": 1, "kind": "reference",
            "sample": f"{n} full decode GEMV set steps (10 calls) through the reference MatMulQ "
                      f"(oracle/_ref, registry lookup once, kernel call timed), one thread as the "
                      f"reference runs it, {secs:.1f} s",
            "columns": [
                {"path": "MatMulQ (src/ops/kernels_matmul.cpp:42-74)", "value": round(mq_val, 4),
                 "unit": UNIT, "cores": 1, "steps": n, "seconds": round(secs, 2)},
                {"path": "fp32 gemm_auto on dequantized weights (backends/cpu/gemm.cpp:288-302)",
                 "value": round(ga_val, 4), "unit": UNIT, "cores": ga_threads, "steps": n2,
                 "seconds": round(secs2, 2),
                 "note": "its thread rule gives one thread at M < 32; its NEON kernel is the scalar "
                         "packed fallback on x86-64"}],
            "host_threads": hw}


def _assert_product_not_loaded():
    with open("/proc/self/maps") as f:
        if "libmtrtq" in f.read():
            raise RuntimeError("the reference arm loaded libmtrtq.so")


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built"}))
        return
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    calls, step_bytes = decode_set_calls()
    tasks = cpu_row_tasks(calls)
    threads = max(1, os.cpu_count() or 1)
    run_pool(tasks, threads, steps=max(1, args.warmup))
    n, secs = run_pool(tasks, threads, steps=args.steps)
    _assert_product_not_loaded()
    value = step_bytes * n / secs / 1e9
    sample = (f"each step: the full decode GEMV set as {len(tasks)} row x column-chunk pieces, each the "
              f"reference MatMulQ kernel (oracle/_ref, prepared once, registry lookup) on its slice, "
              f"on {threads} host threads")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
            "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
            "ms_per_step": round(secs / n * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 W -> fp32, fp32 multiply-add (the reference's MatMulQ)",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights quantized per channel)",
            "config": decode_set_config(args, world, step_bytes),
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference_arm(args)
        return
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from mini_tensorrt_b200 import build as _b
    _b.build()
    if args.workload.startswith("shape:"):
        print(json.dumps(run_shape(args, torch, dev)))
        return
    if args.workload == "gpt2_decode":
        if rank == 0:
            print(json.dumps({"metric": METRIC, "impl": "ours", "n_gpus": 1, **run_gpt2_decode(args, torch, dev)}))
        return
    if args.workload == "tp_decode":
        line = run_tp_decode(args, torch, rank, world, dev, dist)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line))
        return
    if args.workload.startswith("sharded:"):
        line = run_sharded(args, torch, rank, world, dev, dist)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line))
        return
    sharded_line = None
    if world > 1 and args.multi == "sharded":
        sharded_line = run_sharded_decode_set(args, torch, rank, world, dev, dist)
        torch.cuda.empty_cache()
    line, calls, stream = run_ours(args, torch, rank, world, dev, dist)
    del calls
    torch.cuda.empty_cache()
    if sharded_line is not None:
        # headline: the strong-scaled decode set; the replicas (each rank its own
        # full set, no exchange) stay as a secondary figure
        replicas = {k: line[k] for k in ("value", "ms_per_step", "roofline", "e2e", "gpu_launches")}
        replicas["scaling"] = "weak"
        line.update({k: v for k, v in sharded_line.items() if k != "rank0_weight_bytes_per_step"})
        line["config"]["parallelism"] = f"column-sharded x{world} (strong scaling, peer-memory all-gather)"
        line["method"]["step_launch"] = ("per rank: one mtrtq_gemv_group launch over its column shards, then "
                                         "mtrtq_shard_allgather of the output segments; one CUDA graph per step")
        line["method"]["replicas"] = replicas
        line["roofline"]["scope"] = "the grouped GEMV on one full set (measured in the replicas run)"
        line["e2e"]["scope"] = "replicas: each rank its own full set through the grouped API with host buffers"
        line["method"]["rank0_weight_bytes_per_step"] = sharded_line["rank0_weight_bytes_per_step"]
    if rank == 0 and world == 1 and not args.no_extras:
        line["extras"] = run_extras(torch, dev, args, stream)
        line["extras"]["gpt2_small_decode"] = run_gpt2_decode(args, torch, dev, mode="fp32")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_calls, cpu_bytes = decode_set_calls()
        line["cpu_baseline"] = cpu_baseline_line(cpu_calls, cpu_bytes)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
