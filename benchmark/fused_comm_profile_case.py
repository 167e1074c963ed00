"""Single-GPU cases of the fused communication kernels, for ncu captures and
CUDA-event timing of their host-link leg and compute overlap.

ncu is not run on multi-rank commands on this pool, so the NVLink leg of
these kernels is timed with CUDA events by benchmark/layer_comm_bench.py;
here each kernel runs with world = 1 (its own unit is the only "peer"; the
signal handshake is with itself), which leaves exactly the host leg:

  rs_d2h   fused_rs_d2h over one Llama-3.1-8B decoder layer (218,112,000
           bf16 gradient elements): read from HBM, x 1/N, bf16 stores
           straight into page-locked host memory over PCIe
  ag_qkv   fused_ag_qkv, zero-copy form: the gather warps read the layer's
           bf16 copy from page-locked host memory and store it into the unit
           while the tcgen05 QKV GEMM [4096 x 6144 x 4096] waits for, then
           consumes, its weight rows

    python benchmark/fused_comm_profile_case.py <rs_d2h|ag_qkv> [--time]

Without --time each kernel runs 3 times (ncu captures one with -k/-c).
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from test1_b200 import _native  # noqa: E402

P = 218_112_000            # one decoder layer
T, H, NQKV = 4096, 4096, 6144


def setup():
    dev = torch.device("cuda", 0)
    C = _native.cuda()
    unit = torch.empty(P, dtype=torch.bfloat16, device=dev)
    unit.normal_()
    pad = torch.zeros(2 + 64 + 2, dtype=torch.int32, device=dev)  # [0,W) ready, [W,2W) done, AG slots
    ptrs = torch.tensor([unit.data_ptr()], dtype=torch.int64)
    sigs = torch.tensor([pad.data_ptr()], dtype=torch.int64)
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    ag_counters = torch.zeros(65, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    host = torch.empty(P, dtype=torch.bfloat16).pin_memory()
    return C, unit, ptrs, sigs, counter, ag_counters, err, host


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["rs_d2h", "ag_qkv"])
    ap.add_argument("--time", action="store_true")
    a = ap.parse_args()
    C, unit, ptrs, sigs, counter, ag_counters, err, host = setup()
    epoch = [0]
    if a.case == "rs_d2h":
        def run():
            epoch[0] += 1
            C.fused_rs_d2h(ptrs, sigs, 0, 1, 0, P, host, 1.0, epoch[0], counter, err)
        bytes_host, flops = 2 * P, 0.0
    else:
        host.copy_(unit.cpu())
        x = torch.randn(T, H, device="cuda").bfloat16()
        out = torch.empty(T, NQKV, device="cuda", dtype=torch.bfloat16)
        shards = torch.tensor([[0, P]], dtype=torch.int64)

        def run():
            epoch[0] += 1
            C.fused_ag_qkv(x, unit, NQKV, out, ptrs, sigs, shards, 0, 1, host, None, epoch[0], ag_counters,
                           None, None, 1, 0)
        bytes_host, flops = 2 * P, 2.0 * T * NQKV * H
    if not a.time:
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        print(json.dumps({"case": a.case, "err": int(err.item()), "gemm_err": int(C.gemm_check_error(False))}))
        return
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 5
    s.record()
    for _ in range(n):
        run()
    e.record()
    e.synchronize()
    ms = s.elapsed_time(e) / n
    print(json.dumps({"case": a.case, "ms": round(ms, 3), "host_gbs": round(bytes_host / ms / 1e6, 1),
                      "tflops_while_gathering": round(flops / ms / 1e9, 1) if flops else None,
                      "err": int(err.item())}))


if __name__ == "__main__":
    main()
