"""Benchmark of the routed W4A16 MoE layer on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl muse|reference]
                    [--workload cfg4] [--tokens 1,32,256] [--no-cpu-baseline] [--no-secondary]

Metric: MoE layer us/call and achieved HBM GB/s (% of the measured B200 copy
bandwidth) per token count. Default workload: configuration 4 -- large-expert decode (E=256,
top-8, H=7168, I=2048, uniform router, NVFP4 weights from N(0, 0.02); T in {1, 32, 256}), the
configuration BASELINE.json runs on one B200 and then expert-parallel over 2/4/8 GPUs. On one
GPU the line also carries configuration 2 (E=128, H=2048, I=768, T in {1, 4, 16, 32}, the
small-expert decode sweep) as a secondary device-timed block.

A step is one layer call at every token count of the sweep. Each call is a CUDA-graph replay,
preceded (outside its timing) by a 512 MiB write that flushes the L2, and timed with CUDA events
on the launching stream. `value` is the geometric mean over the sweep of the mean us/call;
`per_T` lists each token count. Under torchrun (N > 1) the layer runs expert-parallel: rank r
holds its contiguous block of E/N experts, every rank sees all tokens (the decode layout), the
fp32 shares are summed over NVLink peer memory by the library's own kernel inside the captured
graphs, and times are the max over ranks -- the same call split N ways (strong scaling). Before
timing, every line checks its outputs: on one GPU against the CPU oracle, on N GPUs the
expert-parallel output against the single-GPU layer (itself pinned to the oracle) and every
rank's bits against rank 0's; the process exits non-zero if a check fails.

`--impl reference` times the CPU oracle (the reference's fp32 dequantise-then-accumulate path
restated in numpy, all host cores) on the same workload; rank 0 only.
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
DEFAULT_WORKLOAD = "cfg4"
SECONDARY_WORKLOAD = "cfg2"
PARITY_TOL = 1.5e-2          # checks.compare's tolerance (reference.py:25)
# Prefill workloads: at N > 1 their tokens are split evenly over the ranks (BASELINE cfg5: "T
# split evenly across ranks") and each rank's call is the routed dispatch + partial layer +
# routed reduce-scatter; the other workloads replicate the tokens (decode layout).
PREFILL_WORKLOADS = ("cfg5",)
# ncu per-launch DRAM traffic of the dominant kernel, recorded from the capture summarised in
# profiles/ (read here so the line can carry it next to the algorithmic bytes)
TRAFFIC_FILE = REPO / "profiles" / "traffic.json"


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("muse", "reference"), default="muse")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--tokens", default=None, help="comma list overriding the workload's sweep")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the secondary cfg2 block")
    ap.add_argument("--experts", type=int, default=None,
                    help="profiling size: the workload's shape with this many experts (all local)")
    return ap.parse_args(argv)


def peaks():
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, bf16_tflops_sustained=1400.0, source="fallback")


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


def gather_ranks(world, values: list[float]) -> list[list[float]]:
    """Every rank's list (same length on every rank), rank order."""
    if world == 1:
        return [values]
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [o.tolist() for o in out]


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

def sweep(synth, name: str, tokens_arg: str | None, experts: int | None = None):
    shape = synth.CONFIGS[name]
    if experts:   # a profiling-sized copy of the workload: same H, I, K and router, fewer experts
        import dataclasses
        shape = dataclasses.replace(shape, n_experts=experts, local_start=0, local_count=None)
    tokens = tuple(int(t) for t in tokens_arg.split(",")) if tokens_arg else synth.TOKENS[name]
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


def published_ratio(name, tokens, value):
    """value / the published geomean over the same token counts, when the workload has one."""
    pub = PUBLISHED_US.get(name)
    if not pub or any(t not in pub for t in tokens):
        return None
    return round(value / geomean([pub[t] for t in tokens]), 4)


def numpy_weights(w):
    return {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else
                v.view(torch.uint16) if v.dtype == torch.bfloat16 else v).cpu().numpy() for k, v in w.items()}


def metric_name(name):
    return f"MoE layer us/call (geomean over the token sweep), {name}"


def shard(inp: dict, rank: int, world: int) -> dict:
    """This rank's contiguous slice of a batch (T divisible by the rank count)."""
    t = inp["hidden_states"].shape[0]
    if t % world:
        raise SystemExit(f"T={t} is not divisible by {world} ranks")
    lo, hi = rank * t // world, (rank + 1) * t // world
    return {k: (v[lo:hi] if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


def config_block(name, shape, tokens, n_gpus):
    return {"workload": f"{name}: E={shape.n_experts} top-{shape.top_k} H={shape.hidden} "
                        f"I={shape.inter} local=[{shape.local_start},{shape.local_start + shape.n_local}) "
                        f"router={shape.router} T={list(tokens)}",
            "weights": ("NVFP4 from the reference's generators (log-normal e4m3 block scales, "
                        "Student-t expert popularity, busiest-rank rotation)"
                        if shape.router.startswith("reference") else
                        "NVFP4 (e2m1, e4m3 block-16 scales, fp32 global scale) from N(0,0.02)"),
            "activations": "bf16 N(0,1)", "l2": "flushed by a 512 MiB write before every timed call",
            "parallelism": ("single GPU" if n_gpus == 1 else
                            f"ep{n_gpus}: experts split in contiguous blocks, tokens split evenly over the "
                            "ranks, token rows dispatched over NVLink peer memory to the ranks owning "
                            "their experts, fp32 shares of those ranks summed back over NVLink"
                            if name in PREFILL_WORKLOADS else
                            f"ep{n_gpus}: experts split in contiguous blocks, tokens replicated, "
                            "fp32 shares summed over NVLink peer memory")}


# ----------------------------------------------------------------------------- reference arm

def run_reference(args, world, rank):
    """The CPU oracle on the same workload, all host cores. Each step is one sweep over the token
    counts; at each count the oracle runs over a bounded sample of the local experts the batch
    hits (at most as many experts as host threads, the lowest ids; the batch's pairs with other
    experts are left out) and its time is scaled by (experts hit) / (experts sampled): the
    oracle's cost is per expert (fp32 dequantisation of its weights dominates), so the scaled
    time estimates the whole call. The whole run ends in about a minute."""
    if rank != 0:
        return 0
    from oracle import moe_oracle as orc

    pkg = __graft_entry__.load_package()
    from muse_moe_w4a16_b200 import synth
    shape, tokens = sweep(synth, args.workload, args.tokens, args.experts)
    cores = os.cpu_count() or 1
    w_np = numpy_weights(make_weights(synth, shape, "cuda" if torch.cuda.is_available() else "cpu"))
    del pkg
    inputs = {t: make_input(synth, shape, args.workload, t) for t in tokens}
    lo, cnt = shape.local_start, shape.n_local
    samples = {}
    for t in tokens:
        ids = inputs[t]["topk_ids"].numpy()
        hit = sorted({int(e) for e in ids.reshape(-1) if lo <= e < lo + cnt})
        keep = hit[:cores]
        masked = np.where(np.isin(ids, keep), ids, -1).astype(np.int32)
        samples[t] = (masked, len(hit) / max(len(keep), 1), len(keep), len(hit))

    def call(t):
        d = inputs[t]
        masked = samples[t][0]
        orc.ref_kernel_threads(d["hidden_states"].view(torch.uint16).numpy(), masked,
                               d["topk_weights"].numpy(), w_np, lo, cnt, shape.inter, threads=cores)

    for _ in range(args.warmup):
        for t in tokens:
            call(t)
    per_step, per_t_samples = [], {t: [] for t in tokens}
    for _ in range(args.steps):
        step_us = 0.0
        for t in tokens:
            t0 = time.perf_counter()
            call(t)
            us = (time.perf_counter() - t0) * 1e6 * samples[t][1]
            per_t_samples[t].append(us)
            step_us += us
        per_step.append(step_us)
    per_t = {t: statistics.mean(v) for t, v in per_t_samples.items()}
    value = geomean(list(per_t.values()))
    sample_txt = ("each step: one oracle call per token count over a sample of the experts hit "
                  + ", ".join(f"T={t}: {samples[t][2]} of {samples[t][3]}" for t in tokens)
                  + f" ({cores} threads), times scaled by experts hit / experts sampled")
    line = {
        "impl": "reference", "metric": metric_name(args.workload), "value": value, "unit": "us/call",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(per_step) / 1e3, "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args.workload, shape, tokens, args.gpus),
        "per_T": [{"T": t, "us": per_t[t], "experts_sampled": samples[t][2], "experts_hit": samples[t][3]}
                  for t in tokens],
        "cpu_baseline": {"value": value, "unit": "us/call", "cores": cores, "kind": "port",
                         "sample": sample_txt},
        "e2e": {"value": value, "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- CPU baseline leg

def cpu_baseline(shape, tokens, w_np, inputs):
    """The oracle over the whole sweep (all host threads); also returns its outputs, which the
    single-GPU line's parity check compares against."""
    from oracle import moe_oracle as orc
    cores = os.cpu_count() or 1
    per_t, outs = {}, {}
    for t in tokens:
        d = inputs[t]
        t0 = time.perf_counter()
        outs[t] = orc.ref_kernel_threads(d["hidden_states"].cpu().view(torch.uint16).numpy(),
                                         d["topk_ids"].cpu().numpy(), d["topk_weights"].cpu().numpy(), w_np,
                                         shape.local_start, shape.n_local, shape.inter, threads=cores)
        per_t[t] = (time.perf_counter() - t0) * 1e6
    return {"value": geomean(list(per_t.values())), "unit": "us/call", "cores": cores, "kind": "port",
            "sample": f"one call per token count {list(tokens)} (numpy oracle, {cores} threads)",
            "per_T_us": {str(t): v for t, v in per_t.items()}}, outs


# ----------------------------------------------------------------------------- our arm

class _Eager:
    """Stands in for a captured graph: replay() launches the call eagerly."""

    def __init__(self, fn):
        self.fn = fn

    def replay(self):
        self.fn()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint16).numpy()


class Bench:
    def __init__(self, args, world, rank, local):
        self.args, self.world, self.rank, self.local = args, world, rank, local
        self.pkg = __graft_entry__.load_package()
        from muse_moe_w4a16_b200 import _lib, synth, traffic
        self._lib, self.synth, self.traffic = _lib, synth, traffic
        self.dev = torch.device("cuda", local)
        self.flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)

    def timed(self, graph_map, tokens, steps, read_flush=False):
        flush_words = self.flush.view(torch.int64)
        sink = torch.zeros((), dtype=torch.int64, device=self.dev)
        ev = {t: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)] for t in tokens}
        for i in range(steps):
            for t in tokens:
                if read_flush:
                    sink.copy_(flush_words.amax())
                else:
                    self.flush.zero_()
                ev[t][i][0].record(self.stream)
                graph_map[t].replay()
                ev[t][i][1].record(self.stream)
        return ev

    def measure(self, name, tokens, full):
        """Time one workload. `full`: also the end-to-end pass, the reference-harness-style
        pass, the CPU baseline and the parity check (the headline workload)."""
        args, world, dev, synth, traffic, _lib, pkg = (self.args, self.world, self.dev, self.synth,
                                                      self.traffic, self._lib, self.pkg)
        shape = sweep(synth, name, None, self.args.experts if name == self.args.workload else None)[0]
        w = make_weights(synth, shape, dev)
        moe = None
        sharded = world > 1 and name in PREFILL_WORKLOADS
        if world > 1:
            # expert-parallel: this rank repacks and computes only its block of experts; every
            # rank holds all tokens (decode layout) or its slice of them (prefill layout); the
            # exchanges run over NVLink peer memory
            from muse_moe_w4a16_b200 import ep
            moe = ep.ExpertParallelMoE(w)
            if sharded:
                layer_call = moe.forward_sharded
            else:
                moe.reserve_decode(max(tokens), shape.hidden, dev)   # before any graph is captured
                layer_call = moe.forward_replicated
            n_local = len(moe.experts)
        else:
            state = pkg.prepare(w)
            layer_call = lambda d: pkg.kernel_fn(d, state)  # noqa: E731
            n_local = shape.n_local
        inputs = {t: make_input(synth, shape, name, t) for t in tokens}
        # what this rank's calls see: the whole batch, or its slice of it (prefill layout)
        run_in = {t: shard(inputs[t], self.rank, world) for t in tokens} if sharded else inputs

        graphs, outs, dev_in = {}, {}, {}
        for t in tokens:
            d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in run_in[t].items()}
            dev_in[t] = d
            outs[t] = layer_call(d)          # eager first call (kernel attributes, exchange buffers)
            torch.cuda.synchronize()
            if world == 1:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    outs[t] = layer_call(d)
            elif sharded:
                g = _Eager(lambda d=d: layer_call(d))   # millisecond calls: launch cost is noise
            else:
                g = moe.decode_graphs(d)
            graphs[t] = g

        parity = None
        if full and sharded:
            parity = self.parity_sharded(w, tokens, dev_in, layer_call)
        elif full and world > 1:
            parity = self.parity_ep(shape, w, tokens, dev_in, graphs)
        w_np = numpy_weights(w) if (full and world == 1 and not args.no_cpu_baseline) else None
        del w

        self.timed(graphs, tokens, args.warmup)
        torch.cuda.synchronize()
        clocks = None
        if full:
            with ClockSampler(self.local) as sampler:
                barrier(world)
                torch.cuda.synchronize()
                ev = self.timed(graphs, tokens, args.steps)
                torch.cuda.synchronize()
                barrier(world)
            clocks = sampler.summary()
        else:
            barrier(world)
            ev = self.timed(graphs, tokens, args.steps)
            torch.cuda.synchronize()
        per_t = max_over_ranks(world, [statistics.mean(a.elapsed_time(b) * 1e3 for a, b in ev[t]) for t in tokens])
        gpu_out = None
        if full and world == 1:   # the outputs the parity check compares (one more replay each)
            gpu_out = {}
            for t in tokens:
                graphs[t].replay()
                torch.cuda.synchronize()
                gpu_out[t] = bits(outs[t])

        res = {"name": name, "shape": shape, "tokens": tokens, "per_t": per_t, "inputs": inputs,
               "n_local": n_local, "clocks": clocks, "parity": parity}
        if full:
            res["e2e"] = self.e2e(run_in, shape, tokens, layer_call)
        if full and world == 1:
            res["ref_style"] = self.reference_style(graphs, tokens)
        if world == 1:
            res["stage_us"] = self.stages(tokens, dev_in, state, outs)
        elif full and not sharded:
            res["rank_split"] = self.rank_split(tokens, dev_in, moe)
        del graphs
        torch.cuda.synchronize()
        if w_np is not None:
            cpu, ref_outs = cpu_baseline(shape, tokens, w_np, inputs)
            res["cpu_baseline"] = cpu
            res["parity"] = self.parity_oracle(tokens, gpu_out, ref_outs)
        return res

    # -- checks -----------------------------------------------------------------------------

    def parity_oracle(self, tokens, gpu_out, ref_outs):
        from oracle import moe_oracle as orc
        rows = {}
        for t in tokens:
            ok, _, err, worst = orc.compare(gpu_out[t], ref_outs[t], PARITY_TOL)
            rows[str(t)] = {"rel_l2": float(err), "worst_row": float(worst), "ok": bool(ok)}
        return {"against": "CPU oracle (numpy restatement of reference.py:93-107), every row",
                "tol": PARITY_TOL, "per_T": rows, "ok": all(r["ok"] for r in rows.values())}

    def parity_ep(self, shape, w, tokens, dev_in, graphs):
        """Expert-parallel output (a graph replay) against the single-GPU layer on rank 0, and
        every rank's bits against rank 0's."""
        from oracle import moe_oracle as orc
        world, rank, pkg = self.world, self.rank, self.pkg
        state = pkg.prepare(w) if rank == 0 else None
        rows = {}
        all_ok = True
        for t in tokens:
            got = graphs[t].replay()
            torch.cuda.synchronize()
            ref0 = got.clone()                       # bf16 (a byte copy through NCCL)
            torch.distributed.broadcast(ref0, 0)
            same = torch.equal(got.view(torch.int16), ref0.view(torch.int16))
            equal = torch.tensor([1 if same else 0], dtype=torch.int32, device=self.dev)
            torch.distributed.all_reduce(equal, op=torch.distributed.ReduceOp.MIN)
            row = {"ranks_bit_equal": bool(equal.item())}
            if rank == 0:
                single = pkg.kernel_fn(dev_in[t], state)
                torch.cuda.synchronize()
                ok, _, err, worst = orc.compare(bits(got), bits(single), PARITY_TOL)
                row.update({"rel_l2": float(err), "worst_row": float(worst), "ok": bool(ok)})
                all_ok &= ok and row["ranks_bit_equal"]
            rows[str(t)] = row
        del state
        torch.cuda.empty_cache()
        flag = torch.tensor([1 if all_ok else 0], device=self.dev)
        torch.distributed.broadcast(flag, 0)
        self._lib.device_status(reset=True)
        return {"against": "single-GPU layer on rank 0 (pinned to the CPU oracle by the tests); "
                           "every rank's bits against rank 0's",
                "tol": PARITY_TOL, "per_T": rows, "ok": bool(flag.item())}

    def parity_sharded(self, w, tokens, dev_in, layer_call):
        """Prefill layout: every rank's rows against the single-GPU layer on the same tokens
        (all experts, computed on that rank); the worst rank's figures."""
        from oracle import moe_oracle as orc
        pkg = self.pkg
        state = pkg.prepare(w)
        rows, all_ok = {}, True
        for t in tokens:
            got = layer_call(dev_in[t])
            single = pkg.kernel_fn(dev_in[t], state)
            torch.cuda.synchronize()
            ok, _, err, worst = orc.compare(bits(got), bits(single), PARITY_TOL)
            r = gather_ranks(self.world, [float(err), float(worst), 1.0 if ok else 0.0])
            row = {"rel_l2": max(x[0] for x in r), "worst_row": max(x[1] for x in r),
                   "ok": all(x[2] == 1.0 for x in r)}
            all_ok &= row["ok"]
            rows[str(t)] = row
        del state
        torch.cuda.empty_cache()
        self._lib.device_status(reset=True)
        return {"against": "single-GPU layer on each rank's own tokens (pinned to the CPU oracle by the "
                           "tests); worst rank", "tol": PARITY_TOL, "per_T": rows, "ok": all_ok}

    # -- extra passes -----------------------------------------------------------------------

    def e2e(self, inputs, shape, tokens, layer_call):
        """Pinned host inputs -> device, layer call, result -> pinned host, timed per call. One
        end-to-end graph is built, timed and released at a time."""
        args, world, dev, stream = self.args, self.world, self.dev, self.stream
        h2d = sum(inputs[t][k].numel() * inputs[t][k].element_size()
                  for t in tokens for k in ("hidden_states", "topk_ids", "topk_weights"))
        rows = {t: inputs[t]["hidden_states"].shape[0] for t in tokens}   # this rank's tokens
        d2h = sum(rows[t] * shape.hidden * 2 for t in tokens)
        per_t = []
        for t in tokens:
            hi = {k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in inputs[t].items()}
            ho = torch.empty((rows[t], shape.hidden), dtype=torch.bfloat16).pin_memory()
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
            evs = []
            for i in range(max(1, args.warmup) + args.steps):
                self.flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
                if i >= max(1, args.warmup):
                    evs.append((e0, e1))
            torch.cuda.synchronize()
            per_t.append(statistics.mean(a.elapsed_time(b) * 1e3 for a, b in evs))
            del g, hi, ho, d
        per_t = max_over_ranks(world, per_t)
        return {"value": round(geomean(per_t), 3), "unit": "us/call", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "how": ("CUDA graph of " if world == 1 else "eager ") +
                       "pinned-host->device copies, layer call, device->pinned-host copy",
                "per_T_us": {str(t): round(v, 3) for t, v in zip(tokens, per_t)}}

    def reference_style(self, graphs, tokens):
        """The reference harness's way (TASK.md:66-70): L2 emptied by *reading* a buffer larger
        than L2 (clean lines; the headline's write leaves dirty ones that the call must write
        back), and the fixed cost of a graph replay, which that harness subtracts."""
        args, dev = self.args, self.dev
        tiny = torch.zeros(1, dtype=torch.int32, device=dev)
        g_floor = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_floor):
            tiny.add_(1)
        floor_ev = self.timed({t: g_floor for t in tokens}, tokens, args.warmup + args.steps, read_flush=True)
        rd_ev = self.timed(graphs, tokens, args.warmup + args.steps, read_flush=True)
        torch.cuda.synchronize()
        floor_us = statistics.mean(a.elapsed_time(b) * 1e3 for t in tokens for a, b in floor_ev[t][args.warmup:])
        rd = {t: statistics.mean(a.elapsed_time(b) * 1e3 for a, b in rd_ev[t][args.warmup:]) for t in tokens}
        del g_floor
        return {"floor_us": round(floor_us, 3), "us_read_flush": {t: round(v, 3) for t, v in rd.items()}}

    def stages(self, tokens, dev_in, state, outs):
        """Per-kernel times: the same calls, eager, with events recorded between the kernels (the
        512 MiB flush in front of each call keeps the GPU behind the host, so no event waits on
        a launch). [0]->[1] route + gather (empty when GEMM1 routes), [1]->[2] GEMM1,
        [2]->[3] GEMM2, [3]->[4] combine."""
        stage = {t: [] for t in tokens}
        for _ in range(self.args.steps):
            for t in tokens:
                evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
                self.flush.zero_()
                self.pkg.kernel_fn(dev_in[t], state, out=outs[t], stage_events=evs)
                stage[t].append(evs)
        torch.cuda.synchronize()
        return {t: [statistics.mean(e[j].elapsed_time(e[j + 1]) * 1e3 for e in stage[t]) for j in range(4)]
                for t in tokens}

    def rank_split(self, tokens, dev_in, moe):
        """Each rank's time in its layer kernels and in the exchange (which includes the wait for
        the slowest peer's signal), eager calls after an L2 flush, every rank in step."""
        split = {t: [] for t in tokens}
        for _ in range(self.args.steps):
            for t in tokens:
                evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                self.flush.zero_()
                barrier(self.world)
                moe.forward_replicated(dev_in[t], stage_events=evs)
                split[t].append(evs)
        torch.cuda.synchronize()
        flat = []
        for t in tokens:
            flat += [statistics.mean(e[0].elapsed_time(e[1]) * 1e3 for e in split[t]),
                     statistics.mean(e[1].elapsed_time(e[2]) * 1e3 for e in split[t])]
        per_rank = gather_ranks(self.world, flat)
        return {str(t): {"layer_us": [round(r[2 * i], 2) for r in per_rank],
                         "exchange_us": [round(r[2 * i + 1], 2) for r in per_rank],
                         "exchange_mode": moe.exchange_mode(t * dev_in[t]["hidden_states"].shape[1])}
                for i, t in enumerate(tokens)}

    # -- rows -------------------------------------------------------------------------------

    def rows(self, res):
        """Per token count: time, algorithmic bytes and FLOPs, HBM fraction, launch plan and,
        on one GPU, the per-kernel split; plus the dominant kernel's roofline aggregate."""
        shape, tokens, world, traffic, _lib = res["shape"], res["tokens"], self.world, self.traffic, self._lib
        pk = peaks()
        dims = (shape.local_start, shape.n_local, shape.hidden, shape.inter)
        stage_us = res.get("stage_us", {})
        per_rows, dom_bytes, dom_time, launches = [], 0.0, 0.0, 0
        dom_flops = 0.0
        for t, us in zip(tokens, res["per_t"]):
            ids = res["inputs"][t]["topk_ids"].numpy()
            b = traffic.layer_bytes(ids, *dims)
            f = traffic.layer_flops(ids, *dims)
            plan = _lib.launch_plan(t, shape.top_k, res["n_local"], shape.hidden, shape.inter, shape.n_experts)
            launches += plan["launches"] + (1 if world > 1 else 0)   # + the exchange kernel
            gbs = b / (us * 1e-6) / 1e9
            row = {"T": t, "us": round(us, 3), "bytes": b, "flops": f, "GBps": round(gbs, 1),
                   "hbm_frac": round(gbs / (pk["hbm_gbs"] * world), 4),
                   "roofline_us": round(max(b / (pk["hbm_gbs"] * world) / 1e3,
                                            f / (pk["bf16_tflops"] * world) / 1e6), 3),
                   "launches": plan["launches"], "n_box": plan["n_box"], "path": plan["path"]}
            if "ref_style" in res:
                rd = res["ref_style"]["us_read_flush"][t]
                row.update({"us_read_flush": rd,
                            "us_read_flush_minus_floor": round(rd - res["ref_style"]["floor_us"], 3)})
            if t in stage_us:
                pre, k1, k2, comb = stage_us[t]
                if plan["fused"]:
                    row.update({"kernels_us": {"layer": round(k1, 3)},
                                "layer_kernel_GBps": round(b / (k1 * 1e-6) / 1e9, 1)})
                    dom_bytes += b
                    dom_flops += f
                    dom_time += k1
                else:
                    b1 = traffic.gemm1_bytes(ids, *dims)
                    b2 = traffic.gemm2_bytes(ids, *dims)
                    row.update({"kernels_us": {"route_gather": round(pre, 3), "gemm1": round(k1, 3),
                                               "gemm2": round(k2, 3), "combine": round(comb, 3)},
                                "gemm1_GBps": round(b1 / (k1 * 1e-6) / 1e9, 1),
                                "gemm2_GBps": round(b2 / (k2 * 1e-6) / 1e9, 1)})
                    f1 = traffic.gemm1_flops(ids, *dims)
                    row["gemm1_TFLOPs"] = round(f1 / (k1 * 1e-6) / 1e12, 1)
                    dom_bytes += b1
                    dom_flops += f1
                    dom_time += k1
            if "rank_split" in res:
                row["ranks"] = res["rank_split"][str(t)]
            per_rows.append(row)
        return per_rows, dom_bytes, dom_time, launches, dom_flops


def traffic_record(name):
    """ncu DRAM bytes per launch of the dominant kernel for this workload, if recorded."""
    if not TRAFFIC_FILE.exists():
        return None
    return json.loads(TRAFFIC_FILE.read_text()).get(name)


def run_muse(args, world, rank, local):
    b = Bench(args, world, rank, local)
    shape, tokens = sweep(b.synth, args.workload, args.tokens, args.experts)
    res = b.measure(args.workload, tokens, full=True)
    per_rows, dom_bytes, dom_time, launches, dom_flops = b.rows(res)
    per_t = res["per_t"]
    pk = peaks()
    bound, unit = "hbm", "GB/s"
    if world == 1:
        roof_kernel = ("expert_gemm_tc launch of each call's dominant kernel (the single fused "
                       "layer kernel for decode batches, else GEMM1): algorithmic {} per launch / "
                       "mean CUDA-event duration, summed over the token sweep")
        # the bound whose roofline time is longer: weight bytes at HBM bandwidth, or the MMA
        # FLOPs at the sustained bf16 peak (the dominant kernels of prefill run for milliseconds)
        if dom_flops / (pk["bf16_tflops_sustained"] * 1e12) > dom_bytes / (pk["hbm_gbs"] * 1e9):
            bound, unit = "tensor", "TFLOP/s"
            achieved = dom_flops / (dom_time * 1e-6) / 1e12
            roof_peak = pk["bf16_tflops_sustained"]
            roof_kernel = roof_kernel.format("FLOPs") + ", against the sustained bf16 peak"
        else:
            achieved = dom_bytes / (dom_time * 1e-6) / 1e9
            roof_peak = pk["hbm_gbs"]
            roof_kernel = roof_kernel.format("bytes")
    else:
        # whole expert-parallel call: the work of every rank over the slowest rank's time,
        # against N GPUs' peak -- FLOPs for a tensor-bound (prefill) sweep, else bytes
        flops = sum(r["flops"] for r in per_rows)
        nbytes = sum(r["bytes"] for r in per_rows)
        if flops / (pk["bf16_tflops_sustained"] * 1e12) > nbytes / (pk["hbm_gbs"] * 1e9):
            bound, unit = "tensor", "TFLOP/s"
            achieved = flops / (sum(per_t) * 1e-6) / 1e12
            roof_peak = pk["bf16_tflops_sustained"] * world
            what = f"{world} x the sustained bf16 peak"
        else:
            achieved = nbytes / (sum(per_t) * 1e-6) / 1e9
            roof_peak = pk["hbm_gbs"] * world
            what = f"{world} x HBM peak"
        roof_kernel = (f"whole expert-parallel layer call over {world} GPUs (local layer kernels + "
                       f"peer-memory exchanges), sweep aggregate, against {what}")
    tr = traffic_record(args.workload) if world == 1 else None
    line = {
        "metric": metric_name(args.workload), "value": round(geomean(per_t), 3), "unit": "us/call",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(per_t) / 1e3, 5), "higher_is_better": False,
        "scaling": "strong",   # the same calls at every N, the experts split N ways
        "vs_baseline": published_ratio(args.workload, tokens, geomean(per_t)), "dtype": "bf16",
        "data": "synthetic (seeded; random-init NVFP4 weights)",
        "config": config_block(args.workload, shape, tokens, world),
        "per_T": per_rows,
        "roofline": {"bound": bound, "achieved": round(achieved, 1), "peak": roof_peak, "unit": unit,
                     "frac": round(achieved / roof_peak, 4),
                     "traffic": tr["bytes_per_launch"] if tr else None,
                     "peak_source": pk["source"], "kernel": roof_kernel},
        "e2e": res["e2e"],
        "parity": res["parity"],
        "gpu_launches": launches * args.steps,
        "clocks": res["clocks"],
    }
    if tr:
        line["roofline"]["traffic_source"] = tr["source"]
    if "ref_style" in res:
        rd = [res["ref_style"]["us_read_flush"][t] for t in tokens]
        fl = res["ref_style"]["floor_us"]
        line["reference_harness_style"] = {
            "how": "same graphs; L2 emptied by reading (not writing) 512 MiB before each replay; "
                   "floor = replay of a one-kernel graph after the same read",
            "floor_us": fl, "value": round(geomean(rd), 3),
            "value_minus_floor": round(geomean([v - fl for v in rd]), 3)}
    if "cpu_baseline" in res and rank == 0:
        line["cpu_baseline"] = res["cpu_baseline"]
    if (world == 1 and not args.no_secondary and args.workload == DEFAULT_WORKLOAD and args.tokens is None
            and args.experts is None):
        s_shape, s_tokens = sweep(b.synth, SECONDARY_WORKLOAD, None)
        sres = b.measure(SECONDARY_WORKLOAD, s_tokens, full=False)
        s_rows, s_bytes, s_time, _, _ = b.rows(sres)
        line["secondary"] = {SECONDARY_WORKLOAD: {
            "config": config_block(SECONDARY_WORKLOAD, s_shape, s_tokens, world)["workload"],
            "value": round(geomean(sres["per_t"]), 3), "unit": "us/call", "per_T": s_rows,
            "dominant_kernel_hbm_frac": round(s_bytes / (s_time * 1e-6) / 1e9 / pk["hbm_gbs"], 4)}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ok = res["parity"] is None or res["parity"]["ok"]
    return 0 if ok else 3


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
