"""Causal GQA attention: this library's tcgen05 kernels against flash-attn 2
(the reference trains with attn_implementation="flash_attention_2",
config.py:82) on the same GPU, inputs and layout.

    python benchmark/attention_vs_flash.py [--shapes 4x1024,2x4096] [--json out.json]

Also times every forward variant of this library (mode 1: one query tile
per CTA; mode 2: two tiles per CTA with 0, 1 or 2 of every 8 exponentials on
the FMA-pipe polynomial).  Both read q, k and v from one fused [B*S, (Hq + 2 Hkv) * D] bf16 projection
output (flash-attn gets strided [B, S, H, D] views of it, which it accepts
without a copy).  Timed with CUDA events after warm-up, 20 launches per
figure; attention is compute-bound, so no L2 flush is inserted.  FLOPs:
forward 4 * B * Hq * D * S(S+1)/2 (causal), backward 2.5x the forward.
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
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


def peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)["bf16_tflops"], "of measured"
    except Exception:
        return 1590.0, "of fallback"


def run_shape(B, S, Hq=32, Hkv=8, D=128):
    from flash_attn import flash_attn_interface as fi

    tf_peak, tag = peak()
    T = B * S
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda", generator=g).bfloat16()
    scale = D ** -0.5
    o, lse = native.attention_qkv_fwd(qkv, Hq, Hkv, D, S)
    do = torch.randn(T, Hq * D, device="cuda", generator=g).bfloat16()

    v4 = qkv.view(B, S, Hq + 2 * Hkv, D)
    q, k, v = v4[:, :, :Hq], v4[:, :, Hq:Hq + Hkv], v4[:, :, Hq + Hkv:]
    fa_out, fa_lse, _, _ = fi._flash_attn_forward(q, k, v, 0.0, scale, True, -1, -1, 0.0, None, False)
    dq = torch.empty(B, S, Hq, D, device="cuda", dtype=torch.bfloat16)
    dk = torch.empty(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    dv = torch.empty_like(dk)
    do4 = do.view(B, S, Hq, D)

    def fa_fwd():
        fi._flash_attn_forward(q, k, v, 0.0, scale, True, -1, -1, 0.0, None, False)

    def fa_bwd():
        fi._flash_attn_backward(do4, q, k, v, fa_out, fa_lse, dq, dk, dv, 0.0, scale, True, -1, -1, 0.0,
                                None, False, None)

    ours_fwd = timeit(lambda: native.attention_qkv_fwd(qkv, Hq, Hkv, D, S))
    ours_bwd = timeit(lambda: native.attention_qkv_bwd(do, qkv, o, lse, Hq, Hkv, D, S))
    fa_f = timeit(fa_fwd)
    fa_b = timeit(fa_bwd)

    # agreement of the two forwards and backwards (same inputs)
    diff_o = (o.float() - fa_out.reshape(T, Hq * D).float()).abs().max().item()
    dqkv = native.attention_qkv_bwd(do, qkv, o, lse, Hq, Hkv, D, S).view(B, S, Hq + 2 * Hkv, D)
    fa_bwd()
    diff_dq = (dqkv[:, :, :Hq].float() - dq.float()).abs().max().item()
    diff_dk = (dqkv[:, :, Hq:Hq + Hkv].float() - dk.float()).abs().max().item()
    diff_dv = (dqkv[:, :, Hq + Hkv:].float() - dv.float()).abs().max().item()

    fl_f = 4.0 * B * Hq * D * S * (S + 1) / 2
    fl_b = 2.5 * fl_f
    rows = []
    for kind, ours, fa, fl in (("fwd", ours_fwd, fa_f, fl_f), ("bwd", ours_bwd, fa_b, fl_b)):
        rows.append({"kernel": f"attention_{kind}", "B": B, "S": S, "Hq": Hq, "Hkv": Hkv, "D": D,
                     "ours_ms": round(ours, 4), "ours_tflops": round(fl / ours / 1e9, 1),
                     "ours_frac_peak": round(fl / ours / 1e9 / tf_peak, 3),
                     "flash_attn2_ms": round(fa, 4), "flash_attn2_tflops": round(fl / fa / 1e9, 1),
                     "speedup_vs_flash_attn2": round(fa / ours, 3), "peak_ref": tag})
    rows.append({"check": "max_abs_diff vs flash-attn 2", "B": B, "S": S, "o": diff_o, "dq": diff_dq,
                 "dk": diff_dk, "dv": diff_dv})
    # every forward variant of this library on the same inputs
    old = native.attn_get_mode()
    variants = [(1, None)] + ([(2, k) for k in (0, 1, 2)] if S % 256 == 0 else [])
    for mode, poly in variants:
        native.attn_set_mode(mode)
        if poly is not None:
            native.attn_fwd2_set_poly(poly)
        ms = timeit(lambda: native.attention_qkv_fwd(qkv, Hq, Hkv, D, S))
        rows.append({"kernel": "attention_fwd_variant", "B": B, "S": S, "mode": mode, "poly_of_8": poly,
                     "ms": round(ms, 4), "tflops": round(fl_f / ms / 1e9, 1),
                     "frac_peak": round(fl_f / ms / 1e9 / tf_peak, 3), "peak_ref": tag})
    native.attn_fwd2_set_poly(0)
    native.attn_set_mode(old)
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="4x1024,2x4096")
    ap.add_argument("--json", default="")
    args = ap.parse_args()
    out = []
    for sh in args.shapes.split(","):
        B, S = (int(x) for x in sh.split("x"))
        for r in run_shape(B, S):
            print(json.dumps(r), flush=True)
            out.append(r)
    print("attention mode:", native.attn_get_mode(), "gemm error word:", native.gemm_error())
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
