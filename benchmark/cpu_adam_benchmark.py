"""LayerAdam host-kernel benchmark (the reference's benchmark/cpu_adam_benchmark.py
capability): time one optimizer step on a synthetic layer of a model preset
for a sweep of thread counts, report ms, Gparams/s and achieved host memory
bandwidth (bytes actually moved per parameter: fp32 param r/w, fp32 m and v
r/w, bf16 gradient read, bf16 shadow write = 28 B).

    python benchmark/cpu_adam_benchmark.py --model 8B --threads 1,4,8,16 [--layout fp32|split|both] [--json out.json]
    python benchmark/cpu_adam_benchmark.py --model 8B --compare-reference   # also the reference's JIT cpu_adam
    python benchmark/cpu_adam_benchmark.py --model 8B --profile [--iters 20]   # cProfile of LayerAdam.step
    python benchmark/cpu_adam_benchmark.py --model 8B --perf-stat [--iters 20] # hardware counters (perf stat)

The two analysis modes mirror the reference suite's (cpu_adam_benchmark.py:579-718):
``--profile`` runs LayerAdam.step(0) on one synthetic layer under cProfile and
reports the timing spread and the top functions by cumulative time, which
shows how much of a step is Python dispatch against the native kernel;
``--perf-stat`` re-runs this script as a worker under ``perf stat`` (cycles,
instructions, cache and LLC events) and reports its counters, or says why
perf could not run.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from test1_b200 import _native  # noqa: E402

# per-decoder-layer parameter counts: hidden h, intermediate I, heads H, kv heads G (head_dim h/H)
PRESETS = {
    "3B": (3072, 8192, 24, 8),
    "8B": (4096, 14336, 32, 8),
    "14B": (5120, 13824, 40, 8),
    "32B": (5120, 27648, 40, 8),
    "72B": (8192, 29568, 64, 8),
}


def layer_params(h, I, H, G):
    d = h // H
    return h * (H * d) + 2 * h * (G * d) + (H * d) * h + 3 * h * I + 2 * h


def bench_split(n, threads, steps):
    """The engine's layout: split-plane master (bf16 high plane, which is
    also the GPU copy, + 16-bit low plane), fp32 m/v, bf16 gradient: 26 B."""
    h = _native.host()
    h.configure_threads(threads, [])
    hi = torch.empty(n, dtype=torch.bfloat16)
    lo = torch.empty(n, dtype=torch.int16)
    h.f32_to_split(torch.randn(n), hi, lo)
    g = torch.randn(n).bfloat16()
    m = torch.zeros(n)
    v = torch.zeros(n)
    times = []
    for i in range(steps + 1):
        t0 = time.perf_counter()
        h.adam_step_split(hi, lo, g, m, v, i + 1, 1e-5, 0.9, 0.999, 1e-8, 0.01, True, True, 1.0)
        times.append(time.perf_counter() - t0)
    best = min(times[1:])
    return {"layout": "split", "threads": threads, "ms": round(best * 1e3, 2),
            "gparams_s": round(n / best / 1e9, 3), "gb_s": round(n * 26 / best / 1e9, 1), "bytes_per_param": 26}


def bench(n, threads, steps, with_shadow=True, state=torch.float32):
    h = _native.host()
    h.configure_threads(threads, [])
    p = torch.randn(n)
    g = torch.randn(n).bfloat16()
    m = torch.zeros(n, dtype=state)
    v = torch.zeros(n, dtype=state)
    sh = torch.empty(n, dtype=torch.bfloat16) if with_shadow else None
    times = []
    for i in range(steps + 1):
        t0 = time.perf_counter()
        h.adam_step(p, g, m, v, sh, i + 1, 1e-5, 0.9, 0.999, 1e-8, 0.01, True, True, 1.0)
        times.append(time.perf_counter() - t0)
    best = min(times[1:])
    bytes_per = 4 * 2 + state.itemsize * 4 + 2 + (2 if with_shadow else 0)
    return {"layout": "fp32", "threads": threads, "ms": round(best * 1e3, 2), "gparams_s": round(n / best / 1e9, 3),
            "gb_s": round(n * bytes_per / best / 1e9, 1), "bytes_per_param": bytes_per}


def bench_reference(n, steps):
    """The reference's DeepSpeed-derived cpu_adam through its own loader (JIT
    build).  Gradients must be fp32 there (it upcasts bf16 grads itself)."""
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    from optimizer.layer_adam.builder import CPUAdamLoader  # reference module

    mod = CPUAdamLoader().load()
    mod.create_adam(0, 1e-5, 0.9, 0.999, 1e-8, 0.01, True, False)
    p = torch.randn(n)
    g = torch.randn(n)
    m = torch.zeros(n)
    v = torch.zeros(n)
    times = []
    for i in range(steps + 1):
        t0 = time.perf_counter()
        mod.adam_update(0, i + 1, 1e-5, 0.9, 0.999, 1e-8, 0.01, True, p, g, m, v)
        times.append(time.perf_counter() - t0)
    best = min(times[1:])
    return {"impl": "reference", "threads": torch.get_num_threads(), "ms": round(best * 1e3, 2),
            "gparams_s": round(n / best / 1e9, 3), "gb_s": round(n * 28 / best / 1e9, 1)}


def _layer_adam_case(n, threads):
    """One LayerAdam with a single synthetic layer of n fp32 parameters and
    an fp32 gradient, through the public API (the reference suite's case)."""
    from test1_b200.optim.layer_adam import LayerAdam

    _native.host().configure_threads(threads, [])
    opt = LayerAdam(lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, adamw_mode=True,
                    fp32_optimizer_state=True, num_layer=1)
    param = torch.nn.Parameter(torch.randn(n))
    opt.add_layer_params(0, [param])
    param.grad = torch.randn(n)
    return opt, param


def profile_cprofile(n, threads, iters, top=20):
    import cProfile
    import io
    import pstats
    import statistics

    opt, param = _layer_adam_case(n, threads)
    for _ in range(3):
        opt.step(layer_idx=0)
    prof = cProfile.Profile()
    times = []
    prof.enable()
    for _ in range(iters):
        t0 = time.perf_counter()
        opt.step(layer_idx=0)
        times.append(time.perf_counter() - t0)
    prof.disable()
    buf = io.StringIO()
    pstats.Stats(prof, stream=buf).sort_stats("cumulative").print_stats(top)
    ms = [t * 1e3 for t in times]
    return {"mode": "cprofile", "layer_params": n, "threads": threads, "iters": iters,
            "mean_ms": round(statistics.mean(ms), 3), "min_ms": round(min(ms), 3),
            "max_ms": round(max(ms), 3), "std_ms": round(statistics.pstdev(ms), 3),
            "gparams_s": round(n / (min(ms) / 1e3) / 1e9, 3), "profile": buf.getvalue()}


PERF_EVENTS = ("cycles,instructions,cache-references,cache-misses,L1-dcache-loads,"
               "L1-dcache-load-misses,LLC-loads,LLC-load-misses")


def profile_perf(model, threads, iters):
    """perf stat over a worker run of this script (the worker does 3 warm-up
    and ``iters`` timed LayerAdam steps)."""
    import shutil
    import subprocess

    if shutil.which("perf") is None:
        return {"mode": "perf_stat", "unavailable": "perf is not installed on this host"}
    cmd = ["perf", "stat", "-x", ",", "-e", PERF_EVENTS, sys.executable, os.path.abspath(__file__),
           "--worker", "--model", model, "--threads", str(threads), "--iters", str(iters)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"mode": "perf_stat", "unavailable": "perf stat run timed out"}
    counters = {}
    for line in r.stderr.splitlines():
        parts = line.split(",")
        if len(parts) >= 3 and parts[0].strip().replace(".", "").isdigit():
            counters[parts[2].strip()] = float(parts[0])
    if not counters:
        return {"mode": "perf_stat", "unavailable": (r.stderr.strip().splitlines() or ["no output"])[-1]}
    out = {"mode": "perf_stat", "threads": threads, "iters": iters, "counters": counters}
    if counters.get("cycles"):
        out["ipc"] = round(counters.get("instructions", 0.0) / counters["cycles"], 3)
    if counters.get("LLC-loads"):
        out["llc_miss_rate"] = round(counters.get("LLC-load-misses", 0.0) / counters["LLC-loads"], 4)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="8B", choices=sorted(PRESETS))
    ap.add_argument("--threads", default="")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--json", default="")
    ap.add_argument("--compare-reference", action="store_true")
    ap.add_argument("--layout", default="both", choices=["fp32", "split", "both"])
    ap.add_argument("--profile", action="store_true", help="cProfile of LayerAdam.step on one layer")
    ap.add_argument("--perf-stat", action="store_true", help="hardware counters of LayerAdam.step (perf stat)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--worker", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    n = layer_params(*PRESETS[args.model])
    ncpu = len(os.sched_getaffinity(0))
    threads = [int(t) for t in args.threads.split(",") if t] or sorted({1, max(1, ncpu // 4), max(1, ncpu // 2), ncpu})
    if args.worker:  # the process perf stat measures
        opt, _ = _layer_adam_case(n, threads[-1])
        for _ in range(3 + args.iters):
            opt.step(layer_idx=0)
        return
    if args.profile or args.perf_stat:
        res = []
        if args.profile:
            r = profile_cprofile(n, threads[-1], args.iters)
            print(r.pop("profile"))
            res.append(r)
        if args.perf_stat:
            res.append(profile_perf(args.model, threads[-1], args.iters))
        for r in res:
            print(json.dumps(r), flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(res, f, indent=1)
        return
    res = {"model": args.model, "layer_params": n, "simd": _native.host().simd_level(), "runs": []}
    for t in threads:
        for layout in (("fp32", "split") if args.layout == "both" else (args.layout,)):
            r = bench(n, t, args.steps) if layout == "fp32" else bench_split(n, t, args.steps)
            res["runs"].append(r)
            print(json.dumps(r), flush=True)
    if args.compare_reference:
        try:
            r = bench_reference(n, args.steps)
        except Exception as exc:
            r = {"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"}
        res["reference"] = r
        print(json.dumps(r), flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
