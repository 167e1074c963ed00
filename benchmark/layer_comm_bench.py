"""Per-layer communication microbenchmark (comparison config 5) for one
Llama-3.1-8B decoder layer (218,112,000 params, bf16 on the GPU), 2..8 GPUs:

  (a) shard fetch: this rank's 1/N shard of the layer's bf16 copy (the high
      plane of the split master, page-locked host memory) -> the whole layer
      on every GPU, then the QKV GEMM on activations [4096 tokens x 4096]:
        staged fused  -- copy-engine H2D of the shard into this rank's unit,
                         then fused_ag_qkv (NVLink broadcast inside the
                         tcgen05 QKV GEMM)
        staged split  -- the same H2D, fused_shard_gather (NVLink broadcast
                         on 32 CTAs), then the QKV GEMM
        zero-copy     -- fused_ag_qkv reading the fp32 master (both planes,
                         4 B/param) from host memory itself
      vs. NCCL path: H2D of the bf16 shard + all_gather_into_tensor + cuBLAS
  (b) gradient reduce-scatter + 1/N scale + copy into the page-locked host
      shard                                  -- fused_rs_d2h
      vs. NCCL path: reduce_scatter_tensor + scale + D2H copy
  (c) LayerAdam host step on this rank's shard of the layer
  (d) the same operations through the reference's own DistributedSync,
      unmodified (shard all-gather + cuBLAS QKV; reduce to rank 0 + D2H)

Roofline per fused path = the slowest of: FLOPs / measured bf16 peak, bytes
crossing PCIe / 55 GB/s (measured per-direction host link on this pool), bytes
crossing NVLink / 770 GB/s per direction per GPU.  Timed with CUDA events after
warm-up; every rank reports, rank 0 prints the max over ranks.

    torchrun --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 benchmark/layer_comm_bench.py
"""
from __future__ import annotations

import json
import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

PCIE_GBS = 55.0
NVLINK_GBS = 770.0


def peak_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)["bf16_tflops"], "of measured"
    except Exception:
        return 1590.0, "of fallback"


def timed(fn, iters=5, warmup=2):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters


def maxr(x):
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _reference_sync(dev):
    """The reference's DistributedSync for shard + gpu_reduce, or None when
    its source is not installed under baseline/_ref."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "distributed_sync.py")):
        return None
    import types

    sys.path.insert(0, ref_dir)
    try:
        from distributed_sync import DistributedSync  # the reference's module
    finally:
        sys.path.remove(ref_dir)
    cfg = types.SimpleNamespace(param_transfer_mode="shard", grad_sync_mode="gpu_reduce", device=dev,
                                dtype=torch.bfloat16)
    return DistributedSync(cfg)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from test1_b200 import _native
    from test1_b200.parallel.fused import SymmetricBuffer
    from test1_b200.runtime.host_memory import HostRegion
    from test1_b200.runtime.layer_state import shard_bounds, shard_size

    C = _native.cuda()
    H, I, Hq, Hkv, D = 4096, 14336, 32, 8, 128
    n_qkv = (Hq + 2 * Hkv) * D
    P = H * n_qkv + Hq * D * H + 3 * H * I + 2 * H
    T = 4096
    peak, tag = peak_tflops()
    s, e = shard_bounds(P, world, rank)
    n = e - s
    ss = shard_size(P, world)

    # host shard of the split master, page-locked and mapped
    region = HostRegion(4 * n + 4096)
    hi = region.view(torch.bfloat16, 0, n)
    lo = region.view(torch.int16, 2 * n, n)
    _native.host().f32_to_split(torch.randn(n) * 0.02, hi, lo)
    region.pin([(0, 4 * n)])
    grad_host = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)

    unit = SymmetricBuffer(world * ss, torch.bfloat16, dev, dist.group.WORLD)
    gbuf = SymmetricBuffer(world * ss, torch.bfloat16, dev, dist.group.WORLD)
    gbuf.tensor.normal_()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    shards = torch.tensor([list(shard_bounds(P, world, q)) for q in range(world)], dtype=torch.int64)
    x = torch.randn(T, H, device=dev).bfloat16()
    qkv = torch.empty(T, n_qkv, device=dev, dtype=torch.bfloat16)

    def fused_a():  # zero-copy: the kernel reads both master planes from host memory
        C.fused_ag_qkv(x, unit.tensor, n_qkv, qkv, unit.ptrs, unit.sigs, shards, rank, world,
                       hi, lo, unit.next_epoch(), unit.ag_counters)

    def staged_fused_a():
        unit.tensor[s:e].copy_(hi, non_blocking=True)
        C.fused_ag_qkv(x, unit.tensor, n_qkv, qkv, unit.ptrs, unit.sigs, shards, rank, world,
                       unit.tensor[s:e], None, unit.next_epoch(), unit.ag_counters)

    def staged_split_a():
        unit.tensor[s:e].copy_(hi, non_blocking=True)
        C.fused_shard_gather(unit.ptrs, unit.sigs, rank, world, s, n, unit.tensor[s:e], None,
                             unit.next_epoch(), unit.counter, err, 32)
        C.gemm_bf16(x, unit.tensor[: n_qkv * H].view(n_qkv, H), qkv, False, False, None)

    gathered = torch.empty(world * ss, device=dev, dtype=torch.bfloat16)

    def nccl_a():
        mine = gathered[rank * ss:(rank + 1) * ss]
        mine[:n].copy_(hi, non_blocking=True)
        dist.all_gather_into_tensor(gathered, mine)
        torch.matmul(x, gathered[: n_qkv * H].view(n_qkv, H).t(), out=qkv)

    def fused_b():
        C.fused_rs_d2h(gbuf.ptrs, gbuf.sigs, rank, world, s, n, grad_host, 1.0 / world,
                       gbuf.next_epoch(), gbuf.counter, err)

    rs_out = torch.empty(ss, device=dev, dtype=torch.bfloat16)

    def nccl_b():
        dist.reduce_scatter_tensor(rs_out, gbuf.tensor[: world * ss])
        rs_out.mul_(1.0 / world)
        grad_host[:n].copy_(rs_out[:n], non_blocking=True)

    ta = maxr(timed(fused_a))
    tsa = maxr(timed(staged_fused_a))
    tsp = maxr(timed(staged_split_a))
    tna = maxr(timed(nccl_a))
    tb = maxr(timed(fused_b))
    tnb = maxr(timed(nccl_b))
    code = int(err.item())

    # (d) the reference's own path on the same layer (its DistributedSync,
    # distributed_sync.py:99-158 and :242-300, run unmodified): H2D of this
    # rank's slice of its pinned bf16 staging copy, a host synchronisation,
    # all_gather into fresh tensors and copies into the unit, then the QKV
    # GEMM by cuBLAS; gradients reduced to rank 0 in full, averaged and copied
    # to host there.  Its per-pass CPU fp32->bf16 cast into the staging copy
    # (layer_state.py:301) is not timed.
    td_a = td_b = None
    ref_sync = _reference_sync(dev) if world > 1 else None
    if ref_sync is not None:
        staging = torch.empty(P, dtype=torch.bfloat16, pin_memory=True)
        staging.copy_(torch.randn(P) * 0.02)
        ref_unit = torch.empty(P, dtype=torch.bfloat16, device=dev)
        ref_grads = torch.randn(P, device=dev).bfloat16()
        ref_host = torch.empty(P, dtype=torch.bfloat16, pin_memory=True)

        def ref_a():
            ref_sync.gather_params_to_gpu(staging, ref_unit, None)
            torch.matmul(x, ref_unit[: n_qkv * H].view(n_qkv, H).t(), out=qkv)

        def ref_b():
            ref_sync.reduce_gradients_to_master(ref_grads, ref_host, None)

        td_a = maxr(timed(ref_a))
        td_b = maxr(timed(ref_b))

    # (c) host LayerAdam on this rank's shard (split master, bf16 grad)
    m = torch.zeros(n)
    v = torch.zeros(n)
    g = torch.randn(n).bfloat16()
    t0 = time.perf_counter()
    for step in range(1, 4):
        _native.host().adam_step_split(hi, lo, g, m, v, step, 1e-5, 0.9, 0.999, 1e-8, 0.01, True, True, 1.0)
    tc = maxr((time.perf_counter() - t0) / 3 * 1e3)

    flops = 2.0 * T * n_qkv * H
    nvl_a = 2.0 * P * (world - 1) / world  # bf16 bytes each GPU receives from peers
    roof_a = max(flops / (peak * 1e12), 4.0 * n / (PCIE_GBS * 1e9), nvl_a / (NVLINK_GBS * 1e9)) * 1e3
    # staged: 2 B/param over PCIe; the host leg and the NVLink leg run one after the other here
    roof_sa = max(flops / (peak * 1e12), 2.0 * n / (PCIE_GBS * 1e9), nvl_a / (NVLINK_GBS * 1e9)) * 1e3
    pcie_b = 2.0 * n
    nvl_b = 2.0 * n * (world - 1)  # each GPU pulls its shard from N-1 peers
    roof_b = max(pcie_b / (PCIE_GBS * 1e9), nvl_b / (NVLINK_GBS * 1e9)) * 1e3
    if rank == 0:
        out = {
            "n_gpus": world, "layer_params": P, "error_word": code,
            "a_staged_fused_ag_qkv_ms": round(tsa, 3), "a_staged_gather_then_gemm_ms": round(tsp, 3),
            "a_staged_roofline_ms": round(roof_sa, 3), "a_staged_frac_of_roofline": round(roof_sa / tsa, 3),
            "a_nccl_h2d_bf16_allgather_cublas_ms": round(tna, 3),
            "a_zero_copy_fp32_master_fused_ms": round(ta, 3), "a_zero_copy_roofline_ms": round(roof_a, 3),
            "a_zero_copy_frac_of_roofline": round(roof_a / ta, 3),
            "b_fused_rs_d2h_ms": round(tb, 3), "b_nccl_reduce_scatter_d2h_ms": round(tnb, 3),
            "b_roofline_ms": round(roof_b, 3), "b_frac_of_roofline": round(roof_b / tb, 3),
            "c_layeradam_shard_ms": round(tc, 2),
            "d_reference_shard_gather_qkv_ms": None if td_a is None else round(td_a, 3),
            "d_reference_reduce_to_rank0_d2h_ms": None if td_b is None else round(td_b, 3),
            "roofline_inputs": {"pcie_gbs": PCIE_GBS, "nvlink_gbs": NVLINK_GBS, "bf16_tflops": peak,
                                "peak_ref": tag},
        }
        print(json.dumps(out), flush=True)
    dist.barrier()
    region.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
