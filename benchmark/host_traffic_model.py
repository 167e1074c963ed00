"""Host-memory traffic per training step, and the step time it implies, for
the layer-sliding engine at N GPUs of one node.

The engine's 1-GPU step is bound by host DRAM traffic (the optimizer and the
weight streams), so this model predicts how full and shard mode scale once
the host bandwidth is known.  Bytes per parameter per step:

  optimizer (split fp32 master, fp32 m/v, bf16 gradient): read 2 + 4 + 8,
  write 4 + 8 = 26, spread over the ranks' shards (26 in total per step);
  bf16 weight reads by the GPUs, forward and backward: full mode every GPU
  reads the whole layer (2 x 2 x N), shard mode each GPU reads its 1/N and
  the rest crosses NVLink (2 x 2 in total);
  gradient writes (gpu_reduce: each rank stores its reduced shard): 2.

    python benchmark/host_traffic_model.py --params 8.03e9 --host-gbs 190 --tokens-per-gpu 4096

``--host-gbs`` is what the host sustains with everything running (the 1-GPU
step of the Llama-3.1-8B config measured ~190 GB/s on the B200 box).  The
printed step times are predictions, not measurements.  Against the measured
config-2 steps (full mode) at 190 GB/s: 1 GPU 1.35 s predicted / 1.40-1.48 s
measured, 2 GPUs 1.52 / 1.53-1.54, 4 GPUs 1.86 / 1.78, 8 GPUs 2.43 / 2.48.  Shard
mode at 8 GPUs with 8192 tokens per GPU (config 3) measured 1.66 s against 1.35 s
of host traffic: there the GPU work per step (twice the tokens, activation
offload) is no longer hidden entirely.  Shard mode at 2 GPUs
measured 1.77 s against 1.35 predicted: there each layer's fused gather sits
on the forward's critical path (it feeds the QKV GEMM directly instead of
being prefetched a layer ahead), a latency this traffic model leaves out.
"""
from __future__ import annotations

import argparse
import json

OPT_BYTES = 26.0
GRAD_BYTES = 2.0
WEIGHT_PASSES = 2  # forward and the backward reload


def bytes_per_param(n_gpus: int, mode: str) -> float:
    weights = 2.0 * WEIGHT_PASSES * (n_gpus if mode == "full" else 1)
    return OPT_BYTES + weights + GRAD_BYTES


def predict(params: float, host_gbs: float, tokens_per_gpu: int, gpus=(1, 2, 4, 8)) -> list:
    out = []
    for n in gpus:
        for mode in ("full", "shard"):
            if n == 1 and mode == "shard":
                continue
            b = bytes_per_param(n, mode) * params
            t = b / (host_gbs * 1e9)
            out.append({"gpus": n, "mode": mode, "host_gb_per_step": round(b / 1e9, 1),
                        "step_s": round(t, 3), "tokens_per_s": round(n * tokens_per_gpu / t, 1)})
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--params", type=float, default=8.03e9)
    ap.add_argument("--host-gbs", type=float, default=190.0)
    ap.add_argument("--tokens-per-gpu", type=int, default=4096)
    a = ap.parse_args()
    for row in predict(a.params, a.host_gbs, a.tokens_per_gpu):
        print(json.dumps(row))


if __name__ == "__main__":
    main()
