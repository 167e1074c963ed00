"""Per-layer gradient check of the reference's training step (diagnosis tool,
not a benchmark).

Runs the unmodified reference SlideFSDP (baseline/_ref) through its public
API on one GPU and records, at every LayerAdam update, what gradient each
layer hands to the optimizer: elements that are non-finite, the fraction
that is exactly zero, and the largest magnitude.  It wraps the reference's
`LayerAdam.step_with_grad_views` (layer_adam.py:359-425) to observe its
arguments and then calls it unchanged.

    python baseline/reference_grad_check.py [--model tiny|llama31_8b] [--init cpu|cuda] [--steps 3]

What it shows (measured on a B200, tiny model): the last decoder layer's
gradient is exactly zero at step 1 (zero_frac 1.0) and equals a stale buffer
afterwards.  That layer stays resident between its forward and backward, so
its backward fetch returns early (layer_state.py:285-287) and neither zeroes
the pool unit's gradient buffer nor points `param.grad` at it; the copy to
the host (layer_state.py:367-381) reads a buffer the backward never wrote.
With `--init cuda` on the 8B model, that buffer held leftovers of the
GPU-side random initialisation, whose bf16 reinterpretation includes NaN
patterns, which is why an earlier harness saw NaN losses after step 1.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", choices=["tiny", "llama31_8b"])
    ap.add_argument("--init", default="cpu", choices=["cpu", "cuda"])
    ap.add_argument("--steps", type=int, default=3)
    args = ap.parse_args()

    import torch

    from baseline.reference_arm import REF, build_hf_model

    sys.path.insert(0, REF)
    import optimizer.layer_adam.layer_adam as ref_adam  # reference module
    from config import SlideFSDPConfig as RefConfig
    from slide_fsdp import SlideFSDP as RefSlideFSDP

    seen = []
    inner = ref_adam.LayerAdam.step_with_grad_views

    def observed(self, layer_idx=None, grad_views=None, closure=None):
        bad = zero = total = 0
        amax = 0.0
        for g in (grad_views or {}).values():
            f = g.float()
            fin = torch.isfinite(f)
            bad += int((~fin).sum())
            zero += int((f == 0).sum())
            total += f.numel()
            if bool(fin.any()):
                amax = max(amax, float(f[fin].abs().max()))
        seen.append({"layer": layer_idx, "nonfinite": bad, "zero_frac": round(zero / max(total, 1), 4),
                     "absmax": amax})
        return inner(self, layer_idx, grad_views, closure)

    ref_adam.LayerAdam.step_with_grad_views = observed

    dev = torch.device("cuda", 0)
    model, attn = build_hf_model(args.model, dev if args.init == "cuda" else "cpu")
    seq = 128 if args.model == "tiny" else 1024
    cfg = RefConfig(dtype=torch.bfloat16, device=dev, param_transfer_mode="full",
                    grad_sync_mode="gpu_reduce", gpu_buffer_pool_size=2, lr=1e-5, weight_decay=0.01,
                    attention_implementation=attn, ac_offload_mode="cpu", max_seq_length=seq,
                    train_batch_size=4)
    engine = RefSlideFSDP(model, cfg)
    n_layers = len(engine.layer_states)
    gen = torch.Generator().manual_seed(1000)
    for step in range(1, args.steps + 1):
        ids = torch.randint(0, model.config.vocab_size, (4, seq), generator=gen).to(dev)
        loss = float(engine(input_ids=ids, labels=ids).loss.detach())
        for st in engine.layer_states:
            st.wait_for_update()
        torch.cuda.synchronize()
        print(json.dumps({"init": args.init, "model": args.model, "step": step, "loss": loss,
                          "last_decoder_layer": n_layers - 2,
                          "layers_with_nonfinite_grad": [(s["layer"], s["nonfinite"]) for s in seen
                                                         if s["nonfinite"]],
                          "per_layer": sorted(seen, key=lambda s: s["layer"])}), flush=True)
        seen.clear()


if __name__ == "__main__":
    main()
