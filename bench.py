"""Benchmark of the routed W4A16 MoE layer on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl muse|reference]
                    [--workload cfg2] [--tokens 1,4,16,32]

Metric: MoE layer us/call and achieved HBM GB/s (% of the measured B200 copy
bandwidth) per token count. Default workload: configuration 2 (decode; E=128, top-8, H=2048,
I=768; T in {1, 4, 16, 32}; uniform router; NVFP4 weights from N(0, 0.02)).

A step is one layer call at every token count of the sweep. Each call is a CUDA-graph
replay of kernel_fn, preceded (outside its timing) by a 512 MiB write that flushes the L2,
and timed with CUDA events on the launching stream. `value` is the geometric mean over the
sweep of the mean us/call; `per_T` lists each token count. Under torchrun (N > 1) the layer
runs expert-parallel: each rank holds E/N experts, every rank sees all tokens (the decode
layout), the fp32 shares are summed over NVLink peer memory by the library's own kernel inside
the captured graphs, and times are the max over ranks (strong scaling: the same call, split N
ways).

`--impl reference` times the CPU oracle (the reference's fp32 dequantise-then-accumulate
path restated in numpy, all host cores) on the same workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import faulthandler
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
import __graft_entry__  # noqa: E402

FLUSH_BYTES = 512 << 20
PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("muse", "reference"), default="muse")
    ap.add_argument("--workload", default="cfg2")
    ap.add_argument("--tokens", default=None, help="comma list overriding the workload's sweep")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args(argv)


def peaks():
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


def geomean(v):
    return math.exp(sum(math.log(x) for x in v) / len(v))


# ----------------------------------------------------------------------------- distributed

def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(world, values: list[float]) -> list[float]:
    if world == 1:
        return values
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- workloads

def workload(args, pkg_synth):
    shape = pkg_synth.CONFIGS[args.workload]
    tokens = tuple(int(t) for t in args.tokens.split(",")) if args.tokens else pkg_synth.TOKENS[args.workload]
    return shape, tokens


def input_seed(workload_name: str, t: int) -> int:
    return 1000 * int(workload_name.removeprefix("cfg") or 0) + t


# The reference's own problem (cfg0: E=256, top-8, H=I=4096, 32 local experts, the reference's
# generators) is the one shape with published numbers: the reference's best H200 run per shape
# (README.md:13-18), keyed by batch size: decode-1/16/32 and verify-8/128/256.
PUBLISHED_US = {"cfg0": {1: 47.5, 16: 120.3, 32: 154.8, 8: 96.8, 128: 246.7, 256: 327.6}}


def make_weights(synth, shape, device):
    if shape.router.startswith("reference"):
        return synth.reference_weights(shape, seed=synth.WEIGHTS_SEED, device=device)
    return synth.baseline_weights(shape, seed=synth.WEIGHTS_SEED, device=device)


def make_input(synth, shape, workload_name: str, t: int):
    if shape.router.startswith("reference"):
        dist = shape.router.split("-", 1)[1] if "-" in shape.router else "normal"
        return synth.reference_input(shape, t, seed=input_seed(workload_name, t), dist=dist)
    return synth.baseline_input(shape, t, seed=input_seed(workload_name, t))


def published_ratio(args, tokens, value):
    """value / the published geomean over the same token counts, when the workload has one."""
    pub = PUBLISHED_US.get(args.workload)
    if not pub or any(t not in pub for t in tokens):
        return None
    return round(value / geomean([pub[t] for t in tokens]), 4)


# ----------------------------------------------------------------------------- reference arm

def run_reference(args, world, rank):
    if rank != 0:
        return 0
    from oracle import moe_oracle as orc

    pkg = __graft_entry__.load_package()
    from muse_moe_w4a16_b200 import synth
    shape, tokens = workload(args, synth)
    cores = os.cpu_count() or 1
    w = make_weights(synth, shape, "cuda" if torch.cuda.is_available() else "cpu")
    w_np = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else
                v.view(torch.uint16) if v.dtype == torch.bfloat16 else v).cpu().numpy() for k, v in w.items()}
    del pkg
    inputs = {t: make_input(synth, shape, args.workload, t) for t in tokens}

    def call(t):
        d = inputs[t]
        orc.ref_kernel_threads(d["hidden_states"].view(torch.uint16).numpy(), d["topk_ids"].numpy(),
                               d["topk_weights"].numpy(), w_np, shape.local_start, shape.n_local,
                               shape.inter, threads=cores)

    for i in range(args.warmup):
        call(tokens[0])
    samples = {t: [] for t in tokens}
    n = max(args.steps, len(tokens))
    for i in range(n):
        t = tokens[i % len(tokens)]
        t0 = time.perf_counter()
        call(t)
        samples[t].append((time.perf_counter() - t0) * 1e6)
    per_t = {t: statistics.mean(v) for t, v in samples.items()}
    value = geomean(list(per_t.values()))
    line = {
        "impl": "reference", "metric": metric_name(args), "value": value, "unit": "us/call",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sum(per_t.values()) / 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args, shape, tokens),
        "per_T": [{"T": t, "us": per_t[t], "samples": len(samples[t])} for t in tokens],
        "cpu_baseline": {"value": value, "unit": "us/call", "cores": cores, "kind": "port",
                         "sample": f"one layer call per step, token counts {list(tokens)} in rotation"},
        "e2e": {"value": value, "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def metric_name(args):
    return f"MoE layer us/call (geomean over the token sweep), {args.workload}"


def config_block(args, shape, tokens):
    return {"workload": f"{args.workload}: E={shape.n_experts} top-{shape.top_k} H={shape.hidden} "
                        f"I={shape.inter} local=[{shape.local_start},{shape.local_start + shape.n_local}) "
                        f"router={shape.router} T={list(tokens)}",
            "weights": ("NVFP4 from the reference's generators (log-normal e4m3 block scales, "
                        "Student-t expert popularity, busiest-rank rotation)"
                        if shape.router.startswith("reference") else
                        "NVFP4 (e2m1, e4m3 block-16 scales, fp32 global scale) from N(0,0.02)"),
            "activations": "bf16 N(0,1)", "l2": "flushed by a 512 MiB write before every timed call",
            "parallelism": (f"ep{args.gpus}: experts split in contiguous blocks, tokens replicated, "
                            "fp32 shares summed over NVLink peer memory") if args.gpus > 1 else "single GPU"}


# ----------------------------------------------------------------------------- CPU baseline leg

def cpu_baseline(shape, tokens, w, inputs):
    from oracle import moe_oracle as orc
    cores = os.cpu_count() or 1
    w_np = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else
                v.view(torch.uint16) if v.dtype == torch.bfloat16 else v).cpu().numpy() for k, v in w.items()}
    per_t = {}
    for t in tokens:
        d = inputs[t]
        t0 = time.perf_counter()
        orc.ref_kernel_threads(d["hidden_states"].cpu().view(torch.uint16).numpy(), d["topk_ids"].cpu().numpy(),
                               d["topk_weights"].cpu().numpy(), w_np, shape.local_start, shape.n_local,
                               shape.inter, threads=cores)
        per_t[t] = (time.perf_counter() - t0) * 1e6
    return {"value": geomean(list(per_t.values())), "unit": "us/call", "cores": cores, "kind": "port",
            "sample": f"one call per token count {list(tokens)} (numpy oracle, {cores} threads)",
            "per_T_us": {str(t): v for t, v in per_t.items()}}


# ----------------------------------------------------------------------------- our arm

class _Eager:
    """Stands in for a captured graph: replay() launches the call eagerly."""

    def __init__(self, fn):
        self.fn = fn

    def replay(self):
        self.fn()


def run_muse(args, world, rank, local):
    pkg = __graft_entry__.load_package()
    from muse_moe_w4a16_b200 import _lib, synth, traffic

    dev = torch.device("cuda", local)
    shape, tokens = workload(args, synth)
    w = make_weights(synth, shape, dev)
    if world > 1:
        # expert-parallel: this rank repacks and computes only its block of experts; every
        # rank holds all tokens (decode layout) and the fp32 shares are all-reduced over NCCL
        from muse_moe_w4a16_b200 import ep
        moe = ep.ExpertParallelMoE(w)
        moe.reserve_decode(max(tokens), shape.hidden, dev)   # before any graph is captured
        layer_call = moe.forward_replicated
        experts = moe.experts
    else:
        state = pkg.prepare(w)
        layer_call = lambda d: pkg.kernel_fn(d, state)  # noqa: E731
        experts = range(shape.local_start, shape.local_start + shape.n_local)
    inputs = {t: make_input(synth, shape, args.workload, t) for t in tokens}
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    # Device-resident inputs and one captured graph per token count (with N > 1 a pair of
    # graphs, one per exchange-buffer parity: the decode call holds no collective library call).
    graphs, outs, dev_in = {}, {}, {}
    for t in tokens:
        d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in inputs[t].items()}
        dev_in[t] = d
        outs[t] = layer_call(d)          # eager first call (kernel attributes, communicator)
        torch.cuda.synchronize()
        if world == 1:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                outs[t] = layer_call(d)
        else:
            g = moe.decode_graphs(d)
        graphs[t] = g

    # End-to-end: pinned host inputs -> device, layer call, result -> pinned host. One graph
    # per token count, built, timed and released in turn (see e2e_time below).
    h2d = sum(inputs[t][k].numel() * inputs[t][k].element_size()
              for t in tokens for k in ("hidden_states", "topk_ids", "topk_weights"))
    d2h = sum(t * shape.hidden * 2 for t in tokens)

    def e2e_graph(t):
        hi = {k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in inputs[t].items()}
        ho = torch.empty((t, shape.hidden), dtype=torch.bfloat16).pin_memory()
        d = {k: (torch.empty_like(v, device=dev) if isinstance(v, torch.Tensor) else v) for k, v in hi.items()}
        for k in ("hidden_states", "topk_ids", "topk_weights"):
            d[k].copy_(hi[k], non_blocking=True)
        layer_call(d)
        torch.cuda.synchronize()

        def e2e_step():
            for k in ("hidden_states", "topk_ids", "topk_weights"):
                d[k].copy_(hi[k], non_blocking=True)
            ho.copy_(layer_call(d), non_blocking=True)

        if world == 1:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                e2e_step()
        else:
            g = _Eager(e2e_step)
        return g, (hi, ho, d)

    def timed(graph_map, steps, read_flush=False):
        ev = {t: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)] for t in tokens}
        for i in range(steps):
            for t in tokens:
                if read_flush:
                    flush_sink.copy_(flush_words.amax())
                else:
                    flush.zero_()
                ev[t][i][0].record(stream)
                graph_map[t].replay()
                ev[t][i][1].record(stream)
        return ev

    flush_words = flush.view(torch.int64)
    flush_sink = torch.zeros((), dtype=torch.int64, device=dev)

    # warm-up (untimed)
    timed(graphs, args.warmup)
    torch.cuda.synchronize()

    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        ev = timed(graphs, args.steps)
        torch.cuda.synchronize()
        barrier(world)
    # One end-to-end graph alive at a time: a process holding the layer graphs plus every
    # token count's end-to-end graph at once (cfg3: T = 128, 256, 512) crashed inside the graph
    # launch on this pool, while any subset ran clean.
    per_t_e2e = []
    for t in tokens:
        g, keep = e2e_graph(t)
        evs = []
        for i in range(max(1, args.warmup) + args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            if i >= max(1, args.warmup):
                evs.append((e0, e1))
        torch.cuda.synchronize()
        per_t_e2e.append(statistics.mean(a.elapsed_time(b) * 1e3 for a, b in evs))
        del g, keep

    # The reference harness's way (TASK.md:66-70), single GPU only: L2 emptied by *reading* a
    # buffer larger than L2 (clean lines; the headline's write leaves dirty ones that the call
    # must write back), and the fixed cost of a graph replay, which that harness subtracts.
    ref_style = {}
    if world == 1:
        tiny = torch.zeros(1, dtype=torch.int32, device=dev)
        g_floor = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_floor):
            tiny.add_(1)
        floor_ev = timed({t: g_floor for t in tokens}, args.warmup + args.steps, read_flush=True)
        rd_ev = timed(graphs, args.warmup + args.steps, read_flush=True)
        torch.cuda.synchronize()
        floor_us = statistics.mean(a.elapsed_time(b) * 1e3 for t in tokens for a, b in floor_ev[t][args.warmup:])
        ref_style = {"floor_us": round(floor_us, 3),
                     "us_read_flush": {t: round(statistics.mean(a.elapsed_time(b) * 1e3 for a, b in rd_ev[t][args.warmup:]), 3)
                                       for t in tokens}}
        del g_floor

    # Per-kernel times: the same calls, eager, with events recorded between the kernels (the
    # 512 MiB flush in front of each call keeps the GPU behind the host, so no event waits on
    # a launch). [0]->[1] route + gather (empty when GEMM1 routes), [1]->[2] GEMM1,
    # [2]->[3] GEMM2, [3]->[4] combine.
    stage_us = {t: [0.0, 0.0, 0.0, 0.0] for t in tokens}
    if world == 1:
        stage = {t: [] for t in tokens}
        for i in range(args.steps):
            for t in tokens:
                evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
                flush.zero_()
                pkg.kernel_fn(dev_in[t], state, out=outs[t], stage_events=evs)
                stage[t].append(evs)
        torch.cuda.synchronize()
        stage_us = {t: [statistics.mean(e[j].elapsed_time(e[j + 1]) * 1e3 for e in stage[t]) for j in range(4)]
                    for t in tokens}

    per_t = [statistics.mean(a.elapsed_time(b) * 1e3 for a, b in ev[t]) for t in tokens]
    per_t = max_over_ranks(world, per_t)
    per_t_e2e = max_over_ranks(world, per_t_e2e)
    flat = max_over_ranks(world, [v for t in tokens for v in stage_us[t]])
    stage_us = {t: flat[4 * i:4 * i + 4] for i, t in enumerate(tokens)}

    pk = peaks()
    dims = (shape.local_start, shape.n_local, shape.hidden, shape.inter)
    per_rows = []
    g1_bytes = g1_time = 0.0
    launches_per_step = 0
    for t, us in zip(tokens, per_t):
        ids = inputs[t]["topk_ids"].numpy()
        b = traffic.layer_bytes(ids, *dims)
        f = traffic.layer_flops(ids, *dims)
        b1 = traffic.gemm1_bytes(ids, *dims)
        b2 = traffic.gemm2_bytes(ids, *dims)
        pre, k1, k2, comb = stage_us[t]
        plan = _lib.launch_plan(t, shape.top_k, len(experts), shape.hidden, shape.inter)
        launches_per_step += plan["launches"] + (1 if world > 1 else 0)   # + the bf16 cast
        fused = plan["fused"]
        gbs = b / (us * 1e-6) / 1e9
        # the dominant kernel: the single layer kernel of a fused call, else GEMM1
        g1_bytes += b if fused else b1
        g1_time += k1
        row = {"T": t, "us": round(us, 3), "bytes": b, "flops": f, "GBps": round(gbs, 1),
               "hbm_frac": round(gbs / (pk["hbm_gbs"] * world), 4),
               "roofline_us": round(max(b / (pk["hbm_gbs"] * world) / 1e3,
                                        f / (pk["bf16_tflops"] * world) / 1e6), 3),
               "launches": plan["launches"], "n_box": plan["n_box"], "path": plan["path"]}
        if ref_style:
            rd = ref_style["us_read_flush"][t]
            row.update({"us_read_flush": rd, "us_read_flush_minus_floor": round(rd - ref_style["floor_us"], 3)})
        if world == 1 and fused:   # per-kernel event times (single-GPU calls only)
            row.update({"kernels_us": {"layer": round(k1, 3)},
                        "layer_kernel_GBps": round(b / (k1 * 1e-6) / 1e9, 1)})
        elif world == 1:
            row.update({"kernels_us": {"route_gather": round(pre, 3), "gemm1": round(k1, 3),
                                       "gemm2": round(k2, 3), "combine": round(comb, 3)},
                        "gemm1_GBps": round(b1 / (k1 * 1e-6) / 1e9, 1),
                        "gemm2_GBps": round(b2 / (k2 * 1e-6) / 1e9, 1)})
        per_rows.append(row)
    if world == 1:
        achieved = g1_bytes / (g1_time * 1e-6) / 1e9
        roof_kernel = ("expert_gemm_tc launch of each call's dominant kernel (the single fused "
                       "layer kernel for decode batches, else GEMM1): algorithmic bytes per launch / "
                       "mean CUDA-event duration, summed over the token sweep")
        roof_peak = pk["hbm_gbs"]
    else:
        # whole expert-parallel call: every rank's algorithmic bytes over the slowest rank's
        # time, against N GPUs' bandwidth
        achieved = sum(r["bytes"] for r in per_rows) / (sum(per_t) * 1e-6) / 1e9
        roof_kernel = (f"whole expert-parallel layer call over {world} GPUs (local layer kernels + "
                       f"peer-memory exchange), sweep aggregate, against {world} x HBM peak")
        roof_peak = pk["hbm_gbs"] * world
    line = {
        "metric": metric_name(args), "value": round(geomean(per_t), 3), "unit": "us/call",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(per_t) / 1e3, 5), "higher_is_better": False,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": published_ratio(args, tokens, geomean(per_t)), "dtype": "bf16",
        "data": "synthetic (seeded; random-init NVFP4 weights)",
        "config": config_block(args, shape, tokens),
        "per_T": per_rows,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": roof_peak, "unit": "GB/s",
                     "frac": round(achieved / roof_peak, 4), "traffic": None,
                     "peak_source": pk["source"], "kernel": roof_kernel},
        "e2e": {"value": round(geomean(per_t_e2e), 3), "unit": "us/call", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "how": ("CUDA graph of " if world == 1 else "eager ") +
                       "pinned-host->device copies, layer call, device->pinned-host copy"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if ref_style:
        rd = [ref_style["us_read_flush"][t] for t in tokens]
        line["reference_harness_style"] = {
            "how": "same graphs; L2 emptied by reading (not writing) 512 MiB before each replay; "
                   "floor = replay of a one-kernel graph after the same read",
            "floor_us": ref_style["floor_us"], "value": round(geomean(rd), 3),
            "value_minus_floor": round(geomean([v - ref_style["floor_us"] for v in rd]), 3)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(shape, tokens, w, inputs)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graphs   # graphs go before the process group
    torch.cuda.synchronize()
    return 0


def main(argv=None):
    faulthandler.enable()   # a crash prints the Python stack of every thread
    args = parse_args(argv)
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            return run_reference(args, world, rank)
        return run_muse(args, world, rank, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
