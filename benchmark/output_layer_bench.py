"""Output layer of the Llama-3.1-8B step (final RMSNorm excluded): lm_head
GEMM + cross-entropy forward/backward + dx and the lm_head weight gradient,
at T = 4096 tokens, V = 128256, H = 4096, in bf16 on one GPU.

  chunked  -- linear_cross_entropy: per chunk of C tokens the lm_head GEMM
              into one [C, V] buffer, the CE forward+backward in place,
              dx = dlogits W, dW += dlogits^T x by the wgrad GEMM's residual
              epilogue (the role of Liger's fused linear cross-entropy in the
              reference, slide_fsdp.py:86-98)
  full     -- the unchunked sequence: [T, V] logits, CE in place, dgrad, wgrad

Timed with CUDA events (10 launches after 3 warm-up); the peak device memory
of each form is reported from torch.cuda.max_memory_allocated around one call.

    python benchmark/output_layer_bench.py [--chunks 1024,2048,4096]
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from test1_b200.ops import native  # noqa: E402


def timeit(fn, iters=10, warmup=3):
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


def peak_bytes(fn):
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    fn()
    torch.cuda.synchronize()
    return torch.cuda.max_memory_allocated() - base


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--chunks", default="1024,2048,4096")
    a = ap.parse_args()
    T, V, H = a.tokens, a.vocab, a.hidden
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(T, H, device="cuda", generator=g)).bfloat16()
    w = (torch.randn(V, H, device="cuda", generator=g) * 0.02).bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda", generator=g)
    dx = torch.empty_like(x)
    dw = torch.zeros_like(w)
    flops = 3 * 2.0 * T * V * H

    def full():
        logits = native.linear_fwd(x, w)
        loss, dl, _ = native.cross_entropy_fwd_bwd(logits, tgt)
        d = native.linear_dgrad(dl, w)
        native.linear_wgrad(dl, x, out=dw)
        return loss, d

    rows = []
    ms = timeit(full)
    rows.append({"form": "full", "ms": round(ms, 3), "tflops": round(flops / ms / 1e9, 1),
                 "peak_extra_bytes": peak_bytes(full)})
    ref_loss, ref_dx = full()
    for c in (int(v) for v in a.chunks.split(",")):
        def chunked(c=c):  # the first chunk's wgrad overwrites dw, later ones accumulate
            return native.linear_cross_entropy(x, w, tgt, dx, dw, c)
        ms = timeit(chunked)
        loss, _ = chunked()
        rows.append({"form": f"chunked_{c}", "ms": round(ms, 3), "tflops": round(flops / ms / 1e9, 1),
                     "peak_extra_bytes": peak_bytes(chunked),
                     "loss_diff_vs_full": abs(float(loss) - float(ref_loss)),
                     "dx_rel_diff_vs_full": float((dx.float() - ref_dx.float()).norm() / ref_dx.float().norm())})
    for r in rows:
        print(json.dumps(r))
    print("gemm error word:", native.gemm_error())


if __name__ == "__main__":
    main()
