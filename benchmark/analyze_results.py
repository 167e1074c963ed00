"""Summarise cpu_adam_benchmark.py JSON results (the reference's
benchmark/analyze_results.py capability): per file and layout, speed-up and
parallel efficiency against the smallest thread count, best bandwidth, and a
side-by-side table of NUMA bindings when the files come from
numa_benchmark.sh (named ``<binding>.json``).  Plots are written when
matplotlib is importable (``--plot out.png``).

    python benchmark/analyze_results.py results/*.json [--plot adam.png]
"""
from __future__ import annotations

import argparse
import json
import os


def load(path):
    with open(path) as f:
        return json.load(f)


def scaling_rows(res):
    rows = []
    by_layout = {}
    for r in res.get("runs", []):
        by_layout.setdefault(r.get("layout", "fp32"), []).append(r)
    for layout, runs in by_layout.items():
        runs = sorted(runs, key=lambda r: r["threads"])
        base = runs[0]
        for r in runs:
            speedup = base["ms"] / r["ms"]
            eff = speedup / (r["threads"] / base["threads"])
            rows.append((layout, r["threads"], r["ms"], r["gparams_s"], r["gb_s"], speedup, eff))
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("files", nargs="+")
    ap.add_argument("--plot", default="")
    args = ap.parse_args()
    summary = {}
    for path in args.files:
        res = load(path)
        name = os.path.splitext(os.path.basename(path))[0]
        print(f"== {name}: model {res.get('model')} layer {res.get('layer_params'):,} params, simd {res.get('simd')}")
        print(f"{'layout':6s} {'thr':>4s} {'ms':>9s} {'Gparam/s':>9s} {'GB/s':>7s} {'speedup':>8s} {'eff':>6s}")
        rows = scaling_rows(res)
        for layout, t, ms, gp, gb, sp, eff in rows:
            print(f"{layout:6s} {t:4d} {ms:9.2f} {gp:9.3f} {gb:7.1f} {sp:8.2f} {eff:6.2f}")
        if "reference" in res:
            print("reference:", json.dumps(res["reference"]))
        summary[name] = rows
    if len(summary) > 1:
        print("== best bandwidth per file (binding comparison)")
        for name, rows in summary.items():
            best = max(rows, key=lambda r: r[4]) if rows else None
            if best:
                print(f"{name:20s} {best[0]:6s} {best[1]:4d} threads  {best[4]:7.1f} GB/s")
    if args.plot:
        try:
            import matplotlib

            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except Exception:
            print("matplotlib not available: no plot")
            return
        fig, ax = plt.subplots()
        for name, rows in summary.items():
            for layout in sorted({r[0] for r in rows}):
                pts = [(r[1], r[4]) for r in rows if r[0] == layout]
                ax.plot([p[0] for p in pts], [p[1] for p in pts], marker="o", label=f"{name}/{layout}")
        ax.set_xlabel("threads")
        ax.set_ylabel("GB/s")
        ax.legend()
        fig.savefig(args.plot)


if __name__ == "__main__":
    main()
