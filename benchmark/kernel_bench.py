"""Micro-benchmarks of the sm_100a kernels against cuBLAS / PyTorch on the
Llama-3.1-8B layer shapes (T = 4096 tokens).  Timed with CUDA events after
warm-up; each timed launch reads operands larger than... (GEMM operands are
re-used, as inside a layer; the report states it).

    python benchmark/kernel_bench.py [--only gemm,norm,...] [--json out.json]
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from test1_b200.ops import native  # noqa: E402


def timeit(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["hbm_gbs"], "of measured"
    except Exception:
        return 1590.0, 6650.0, "of fallback"


def bench_gemm(T=4096, H=4096, I=14336, nq=32, nkv=8, D=128, modes=(0, 1, 2, 3)):
    tf_peak, _, tag = peaks()
    out = []
    shapes = {
        "qkv_fwd": (T, (nq + 2 * nkv) * D, H),
        "o_fwd": (T, H, nq * D),
        "gateup_fwd": (T, 2 * I, H),
        "down_fwd": (T, H, I),
    }
    for name, (M, N, K) in shapes.items():
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        fl = 2 * M * N * K
        dy = torch.randn(M, N, device="cuda").bfloat16()
        dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
        dw = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        cub = timeit(lambda: torch.matmul(x, w.t(), out=y))
        dgc = timeit(lambda: torch.matmul(dy, w, out=dx))
        wgc = timeit(lambda: torch.matmul(dy.t(), x, out=dw))
        for mode in modes:
            # 3 = mode 2 without its stream-K tail
            native.gemm_set_mode(min(mode, 2))
            native.gemm_set_streamk(mode != 3)
            ours = timeit(lambda: native.gemm(x, w, y))
            dg = timeit(lambda: native.gemm(dy, w, dx, False, True))
            wg = timeit(lambda: native.gemm(dy, x, dw, True, True))
            for kind, t, tc in (("fwd", ours, cub), ("dgrad", dg, dgc), ("wgrad", wg, wgc)):
                out.append({"kernel": f"gemm_{name}_{kind}",
                            "mode": {0: "single", 1: "pair", 2: "pair_tma_store", 3: "pair_tma_store_no_streamk"}[mode],
                            "M": M, "N": N, "K": K, "ms": round(t, 4),
                            "tflops": round(fl / t / 1e9, 1), "frac_peak": round(fl / t / 1e9 / tf_peak, 3),
                            "peak_ref": tag, "cublas_ms": round(tc, 4), "vs_cublas": round(tc / t, 3)})
    native.gemm_set_streamk(True)
    native.gemm_set_mode(2)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default="")
    ap.add_argument("--modes", default="0,1,2,3",
                    help="0 single CTA, 1 pairs, 2 pairs + TMA stores (default), 3 = 2 without the stream-K tail")
    args = ap.parse_args()
    res = bench_gemm(modes=tuple(int(m) for m in args.modes.split(",")))
    for r in res:
        print(json.dumps(r))
    print("gemm error word:", native.gemm_error())
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
