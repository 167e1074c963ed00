"""LayerAdam host-kernel benchmark (the reference's benchmark/cpu_adam_benchmark.py
capability): time one optimizer step on a synthetic layer of a model preset
for a sweep of thread counts, report ms, Gparams/s and achieved host memory
bandwidth (bytes actually moved per parameter: fp32 param r/w, fp32 m and v
r/w, bf16 gradient read, bf16 shadow write = 28 B).

    python benchmark/cpu_adam_benchmark.py --model 8B --threads 1,4,8,16 [--layout fp32|split|both] [--json out.json]
    python benchmark/cpu_adam_benchmark.py --model 8B --compare-reference   # also the reference's JIT cpu_adam
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="8B", choices=sorted(PRESETS))
    ap.add_argument("--threads", default="")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--json", default="")
    ap.add_argument("--compare-reference", action="store_true")
    ap.add_argument("--layout", default="both", choices=["fp32", "split", "both"])
    args = ap.parse_args()
    n = layer_params(*PRESETS[args.model])
    ncpu = len(os.sched_getaffinity(0))
    threads = [int(t) for t in args.threads.split(",") if t] or sorted({1, max(1, ncpu // 4), max(1, ncpu // 2), ncpu})
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
