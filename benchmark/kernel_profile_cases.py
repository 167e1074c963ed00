"""Small single-GPU cases of each sm_100a kernel at Llama-3.1-8B layer shapes
(T = 4096 tokens), for ncu captures and CUDA-event timing.

    python benchmark/kernel_profile_cases.py <case> [--time]

Cases: attn_fwd attn_bwd rmsnorm_fwd rmsnorm_bwd swiglu_fwd swiglu_bwd rope
ce embed_fwd embed_bwd.  Each runs its kernel 3 times (ncu captures one with
-k/-c).  --time prints CUDA-event timing, achieved bandwidth/FLOP rate and
the fraction of the measured peaks.
"""
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from test1_b200.ops import native, reference as ref  # noqa: E402

T, H, I, HQ, HKV, D, V, S = 4096, 4096, 14336, 32, 8, 128, 128256, 1024


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["hbm_gbs"], "of measured"
    except Exception:
        return 1590.0, 6650.0, "of fallback"


def make(case):
    """Returns (fn, bytes moved, flops)."""
    bf = torch.bfloat16
    if case in ("attn_fwd", "attn_bwd"):
        qkv = torch.randn(T, (HQ + 2 * HKV) * D, device="cuda").to(bf)
        causal_pairs = S * (S + 1) / 2 * (T // S)
        fl_f = 4.0 * causal_pairs * HQ * D
        if case == "attn_fwd":
            return (lambda: native.attention_qkv_fwd(qkv, HQ, HKV, D, S)), qkv.numel() * 2 + T * HQ * D * 2, fl_f
        o, lse = native.attention_qkv_fwd(qkv, HQ, HKV, D, S)
        do = torch.randn_like(o)
        return (lambda: native.attention_qkv_bwd(do, qkv, o, lse, HQ, HKV, D, S)), \
            (qkv.numel() * 2) * 2 + o.numel() * 2 * 2, fl_f * 2.5
    if case == "rmsnorm_fwd":
        x = torch.randn(T, H, device="cuda").to(bf)
        w = torch.ones(H, device="cuda").to(bf)
        return (lambda: native.rmsnorm_fwd(x, w, 1e-5)), 2 * x.numel() * 2, 0
    if case == "rmsnorm_bwd":
        x = torch.randn(T, H, device="cuda").to(bf)
        w = torch.ones(H, device="cuda").to(bf)
        _, rstd = native.rmsnorm_fwd(x, w, 1e-5)
        dy = torch.randn_like(x)
        r = torch.randn_like(x)
        return (lambda: native.rmsnorm_bwd(dy, x, w, rstd, r)), 4 * x.numel() * 2, 0
    if case == "swiglu_fwd":
        gu = torch.randn(T, 2 * I, device="cuda").to(bf)
        return (lambda: native.swiglu_gu_fwd(gu)), gu.numel() * 2 * 1.5, 0
    if case == "swiglu_bwd":
        gu = torch.randn(T, 2 * I, device="cuda").to(bf)
        da = torch.randn(T, I, device="cuda").to(bf)
        return (lambda: native.swiglu_gu_bwd(da, gu)), gu.numel() * 2 * 2.5, 0
    if case == "rope":
        qkv = torch.randn(T, (HQ + 2 * HKV) * D, device="cuda").to(bf)
        cos, sin = ref.rope_tables(D, S, 500000.0, None, "cuda")
        return (lambda: native.rope_qkv_(qkv, HQ, HKV, D, cos, sin, S)), T * (HQ + HKV) * D * 2 * 2, 0
    if case == "ce":
        logits = torch.randn(T, V, device="cuda").to(bf)
        tgt = torch.randint(0, V, (T,), device="cuda")
        return (lambda: native.cross_entropy_fwd_bwd(logits, tgt)), logits.numel() * 2 * 3, 0
    if case == "embed_fwd":
        w = torch.randn(V, H, device="cuda").to(bf)
        ids = torch.randint(0, V, (T,), device="cuda")
        return (lambda: native.embedding_fwd(ids, w)), T * H * 2 * 2, 0
    if case == "embed_bwd":
        dh = torch.randn(T, H, device="cuda").to(bf)
        ids = torch.randint(0, V, (T,), device="cuda")
        out = torch.empty(V, H, device="cuda", dtype=bf)
        return (lambda: native.embedding_bwd(dh, ids, V, out)), V * H * 2 + T * H * 2, 0
    raise SystemExit(f"unknown case {case}")


def main():
    case = sys.argv[1]
    fn, nbytes, flops = make(case)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if "--time" in sys.argv:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        n = 20
        for _ in range(n):
            fn()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / n
        tf, bw, tag = peaks()
        out = {"case": case, "ms": round(ms, 4), "gb_s": round(nbytes / ms / 1e6, 1),
               "frac_hbm": round(nbytes / ms / 1e6 / bw, 3), "peak_ref": tag}
        if flops:
            out["tflops"] = round(flops / ms / 1e9, 1)
            out["frac_bf16"] = round(flops / ms / 1e9 / tf, 3)
        print(json.dumps(out))
    else:
        print("ok", case)


if __name__ == "__main__":
    main()
