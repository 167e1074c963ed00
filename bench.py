"""Headline benchmark: Llama-3.1-8B-architecture layer-sliding training,
tokens/s over all GPUs (device-timed, max over ranks).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|fsdp]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Config (comparison config 2): Llama-3.1-8B architecture, random-init N(0,0.02)
weights, fp32 master + fp32 Adam state in pinned host memory, bf16 compute,
param_transfer_mode=full, grad_sync_mode=gpu_reduce, gpu_buffer_pool_size=2,
per-GPU batch 4 x 1024 uniform-random tokens, causal LM loss.  Every timed
step runs the full forward, backward and the host AdamW update of all 8.03 B
parameters.  The weights streamed through the GPU each step (about 30 GB of
host-to-device copies) exceed the 126 MB L2 many times over, so no L2 flush
is inserted.

Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Llama-3.1-8B-arch tokens/sec, device-timed max over ranks, at 1/2/4/8 B200"
BASELINE_VALUE = None  # the reference publishes no number for this metric


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference", "fsdp"], default="ours")
    p.add_argument("--model", default="llama31_8b", choices=["llama31_8b", "tiny", "llama_70b"])
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--param-transfer-mode", default="full", choices=["full", "shard"])
    p.add_argument("--grad-sync-mode", default="gpu_reduce", choices=["gpu_reduce", "cpu_reduce"])
    p.add_argument("--pool", type=int, default=2)
    p.add_argument("--ac-offload", default="cpu", choices=["cpu", "nvme", "none"])
    p.add_argument("--master-layout", default="split", choices=["split", "fp32", "bf16"])
    p.add_argument("--state-dtype", default="fp32", choices=["fp32", "bf16"])
    p.add_argument("--baseline-config", type=int, default=2, choices=[2, 3, 4],
                   help="comparison config preset: 2 = 8B full + gpu_reduce, batch 4 x 1024 (default); "
                        "3 = 8B shard + gpu_reduce, AC cpu, batch 2 x 4096; 4 = 70B shard + cpu_reduce, "
                        "batch 1 x 2048, bf16 weights and Adam state in host RAM (fp32 with >= 1.2 TB)")
    p.add_argument("--no-fuse-gather-qkv", action="store_true",
                   help="shard mode: prefetch each layer with the standalone fused gather instead of "
                        "gathering it inside its QKV GEMM")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-trace-step", action="store_true",
                   help="skip the traced (untimed) step whose per-phase busy times go into the detail")
    p.add_argument("--profile-json", default="")
    args = p.parse_args()
    given = {a.split("=")[0] for a in sys.argv[1:] if a.startswith("--")}
    for k, v in baseline_preset(args.baseline_config, host_ram_bytes()).items():
        if "--" + k.replace("_", "-") not in given:  # explicit flags win
            setattr(args, k, v)
    return args


def host_ram_bytes() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def baseline_preset(cfg: int, ram_bytes: int) -> dict:
    """Flag values of comparison configs 3 and 4.  Config 4 (70B) keeps an
    fp32 master and fp32 Adam state when the host has at least 1.2 TB of RAM
    (about 1.1 TB of host state), else bf16 weights and bf16 state."""
    if cfg == 3:
        return dict(model="llama31_8b", param_transfer_mode="shard", grad_sync_mode="gpu_reduce",
                    batch=2, seq=4096, ac_offload="cpu")
    if cfg == 4:
        big = ram_bytes >= 1.2e12
        return dict(model="llama_70b", param_transfer_mode="shard", grad_sync_mode="cpu_reduce",
                    batch=1, seq=2048, ac_offload="cpu", master_layout="split" if big else "bf16",
                    state_dtype="fp32" if big else "bf16")
    return {}


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons of this rank's GPU
    while running.  nvidia-smi's index of the GPU is looked up by PCI bus id
    (CUDA's device index differs from it when only some of the node's GPUs
    are visible); if that lookup fails, the CUDA index is used."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = self.smi_index(gpu_index, self._bus_id(gpu_index), self._smi_bus_table())
        self.rows = []
        self.proc = None

    @staticmethod
    def _bus_id(idx: int):
        try:
            import torch

            p = torch.cuda.get_device_properties(idx)
            return (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
        except Exception:
            return None

    @staticmethod
    def _smi_bus_table() -> str:
        try:
            return subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id", "--format=csv,noheader"],
                                  capture_output=True, text=True, timeout=20).stdout
        except Exception:
            return ""

    @staticmethod
    def smi_index(cuda_index: int, bus, table: str) -> int:
        """nvidia-smi index of the GPU on PCI address ``bus`` (domain, bus,
        device) in ``table`` ("index, bus id" lines), else ``cuda_index``."""
        if bus is not None:
            for line in table.splitlines():
                try:
                    idx, bid = (x.strip() for x in line.split(",", 1))
                    dom, rest = bid.split(":", 1)
                    b, dev = rest.split(":", 1)
                    if (int(dom, 16), int(b, 16), int(dev.split(".")[0], 16)) == tuple(bus):
                        return int(idx)
                except ValueError:
                    continue
        return cuda_index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def merge_clocks(local: dict, world: int) -> dict:
    """Every rank sampled its own GPU; the line reports the slowest GPU's
    median SM clock, the union of throttle reasons over all GPUs, and each
    GPU's own record (a collective: every rank calls it once)."""
    if world == 1 or local is None:
        return local
    import torch.distributed as dist

    recs = [None] * world
    dist.all_gather_object(recs, local)
    meds = [r.get("sm_mhz") for r in recs if r and r.get("sm_mhz") is not None]
    maxes = [r.get("sm_max_mhz") for r in recs if r and r.get("sm_max_mhz") is not None]
    reasons = sorted({x for r in recs if r for x in r.get("reasons", [])})
    return {"sm_mhz": min(meds) if meds else None, "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": reasons, "samples": sum((r or {}).get("samples", 0) for r in recs),
            "per_gpu": recs}


def init_dist(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def run_ours(args, rank, world, local):
    import torch

    from test1_b200 import SlideFSDPConfig
    from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
    from test1_b200.slide_fsdp import SlideFSDP
    from test1_b200.ops import native_launch_count

    dev = torch.device("cuda", local)
    mcfg = getattr(LlamaConfig, args.model)()
    model = LlamaForCausalLM(mcfg, device="meta")
    cfg = SlideFSDPConfig(dtype=torch.bfloat16, device=dev,
                          param_transfer_mode=args.param_transfer_mode,
                          grad_sync_mode=args.grad_sync_mode, gpu_buffer_pool_size=args.pool,
                          lr=1e-5, weight_decay=0.01, ac_offload_mode=args.ac_offload,
                          max_seq_length=args.seq, train_batch_size=args.batch, seed=42,
                          master_layout=args.master_layout, optimizer_state_dtype=args.state_dtype,
                          fuse_gather_qkv=not args.no_fuse_gather_qkv)
    t0 = time.time()
    engine = SlideFSDP(model, cfg)
    init_s = time.time() - t0

    V = mcfg.vocab_size
    g = torch.Generator().manual_seed(1000 + rank)
    n_batches = args.warmup + 2 * args.steps + 1
    batches = [torch.randint(0, V, (args.batch, args.seq), generator=g).pin_memory() for _ in range(n_batches)]
    dev_batches = [b.to(dev) for b in batches]
    torch.cuda.synchronize()

    losses = []
    # warm-up (untimed)
    for i in range(args.warmup):
        out = engine(input_ids=dev_batches[i], labels=dev_batches[i])
        losses.append(float(out.loss))
    engine.wait_for_updates()
    barrier(world)

    # ---- device-timed loop: inputs pre-staged on the device
    sampler = ClockSampler(local)
    sampler.start()
    launches0 = native_launch_count()
    h2d0 = engine.h2d_bytes
    adam0 = engine.updates.busy_s
    blocked0 = engine.updates.blocked_s
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    start.record()
    last = None
    for k in range(args.steps):
        b = dev_batches[args.warmup + k]
        last = engine(input_ids=b, labels=b).loss
    engine.wait_for_updates()
    end.record()
    end.synchronize()
    barrier(world)
    clocks = sampler.stop()
    launches = native_launch_count() - launches0
    dev_ms = start.elapsed_time(end)
    dev_ms = max_over_ranks(dev_ms, world)
    losses.append(float(last))
    h2d_per_step = (engine.h2d_bytes - h2d0) / args.steps
    adam_busy = (engine.updates.busy_s - adam0) / args.steps
    blocked = (engine.updates.blocked_s - blocked0) / args.steps

    # ---- one traced step after the timed region (untimed): per-phase busy
    # time of this rank (copy stream, compute, gradient stream, optimizer)
    phases = None
    if not args.no_trace_step:
        engine.wait_for_updates()
        barrier(world)
        engine.tracer.start(None)
        b = dev_batches[-1]
        losses.append(float(engine(input_ids=b, labels=b).loss))
        engine.wait_for_updates()
        rec = engine.tracer.last or {}
        engine.tracer.stop()
        phases = {"wall_ms": rec.get("wall_ms"), "phase_ms": rec.get("phase_ms"),
                  "max_over_ranks_ms": rec.get("max_over_ranks_ms")}

    # ---- end-to-end loop through the public API: pinned host batch copied
    # in every step, loss read back every step
    e2e = None
    if not args.no_e2e:
        barrier(world)
        t0 = time.perf_counter()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record()
        for k in range(args.steps):
            hb = batches[args.warmup + args.steps + k]
            ids = hb.to(dev, non_blocking=True)
            out = engine(input_ids=ids, attention_mask=None, labels=ids)
            losses.append(out.loss.item())
        engine.wait_for_updates()
        e_end.record()
        e_end.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
        tokens = args.batch * args.seq * world * args.steps
        e2e = {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": "tokens/s",
               "h2d_bytes_per_step": int(args.batch * args.seq * 8),
               "d2h_bytes_per_step": 4,
               "wall_s": round(time.perf_counter() - t0, 3)}
    engine.close()
    return {
        "dev_ms": dev_ms, "e2e": e2e, "clocks": clocks, "launches": launches, "init_s": init_s,
        "init_phases_s": dict(engine.init_times),
        "losses": losses, "h2d_gb_per_step": h2d_per_step / 1e9, "adam_busy_s_per_step": adam_busy,
        "fetch_blocked_on_adam_s_per_step": blocked, "comm": engine.comm.name,
        "traced_step": phases,
    }


def run_reference(args, rank, world, local):
    from baseline.reference_arm import run as ref_run

    return ref_run(args, rank, world, local)


def main():
    args = parse_args()
    if args.impl == "reference":
        # OpenMP reads its thread count when torch loads: set it first, the
        # way the reference's numa_launch.sh does for each rank.
        from baseline.reference_arm import omp_threads_for_rank

        n = omp_threads_for_rank(int(os.environ.get("LOCAL_RANK", "0")),
                                 int(os.environ.get("LOCAL_WORLD_SIZE", "1")),
                                 len(os.sched_getaffinity(0)))
        os.environ["OMP_NUM_THREADS"] = str(n)
        os.environ["MKL_NUM_THREADS"] = str(n)
    rank, world, local = init_dist(args)
    import torch

    if args.impl in ("reference", "fsdp"):
        if args.impl == "reference":
            res = run_reference(args, rank, world, local)
        else:
            from baseline.fsdp_arm import run as fsdp_run

            res = fsdp_run(args, rank, world, local)
        if res.get("unavailable"):
            if rank == 0:
                print(json.dumps({"impl": args.impl, "unavailable": res["unavailable"]}), flush=True)
            return
    else:
        res = run_ours(args, rank, world, local)

    res["clocks"] = merge_clocks(res.get("clocks"), world)
    res["per_rank"] = gather_per_rank(res, world)
    finite = all_finite(res.get("losses", []), world)
    res["losses_finite"] = finite
    line = make_line(args, world, res)
    if rank == 0:
        print(json.dumps(line), flush=True)
        if args.profile_json:
            with open(args.profile_json, "w") as f:
                json.dump(line, f, indent=2)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if not finite and args.impl == "ours":
        # a diverged run is not a measurement
        print(f"[rank {rank}] non-finite loss in this run: {res.get('losses')}", file=sys.stderr, flush=True)
        sys.exit(3)


PER_RANK_KEYS = ("h2d_gb_per_step", "adam_busy_s_per_step", "fetch_blocked_on_adam_s_per_step",
                 "traced_step", "init_s")


def gather_per_rank(res: dict, world: int):
    """Each rank's own step detail (host traffic, optimizer time, per-phase
    busy time of its traced step), gathered on every rank (a collective)."""
    mine = {k: res[k] for k in PER_RANK_KEYS if k in res}
    if world == 1:
        return [mine]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, mine)
    return out


def all_finite(losses, world: int) -> bool:
    """True when every loss of every rank is finite (a collective)."""
    import math

    ok = all(isinstance(x, (int, float)) and math.isfinite(x) for x in losses)
    if world == 1:
        return ok
    import torch
    import torch.distributed as dist

    t = torch.tensor([1.0 if ok else 0.0], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item() > 0)


def make_line(args, world: int, res: dict) -> dict:
    """The one JSON line of a run: ``res`` holds the device-timed
    milliseconds of the timed steps (max over ranks) and the run's details."""
    tokens = args.batch * args.seq * world * args.steps
    value = tokens / (res["dev_ms"] / 1e3)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["dev_ms"] / args.steps, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
        "dtype": "bf16",
        "data": "synthetic uniform-random tokens, random-init N(0,0.02) weights",
        "config": {
            "model": {"llama31_8b": "Llama-3.1-8B architecture",
                      "llama_70b": "Llama-70B architecture"}.get(args.model, args.model),
            "baseline_config": args.baseline_config,
            "master_layout": args.master_layout, "optimizer_state_dtype": args.state_dtype,
            "global_batch": args.batch * world, "seq_len": args.seq,
            "parallelism": f"dp{world}",
            "param_transfer_mode": args.param_transfer_mode, "grad_sync_mode": args.grad_sync_mode,
            "gpu_buffer_pool_size": args.pool, "ac_offload_mode": args.ac_offload,
            **({"fuse_gather_qkv": not args.no_fuse_gather_qkv} if args.param_transfer_mode == "shard" else {}),
            "l2": "no flush: ~30 GB of weights stream host->device per step (>> 126 MB L2)",
        },
        "clocks": res.get("clocks"),
        "e2e": res.get("e2e"),
        "gpu_launches": res.get("launches"),
    }
    if args.impl != "ours":
        line["impl"] = args.impl
        if args.impl == "fsdp":
            line["config"]["parallelism"] = f"fsdp{world} full_shard, CPU-offloaded params, torch AdamW"
    extra = {k: res[k] for k in ("init_s", "init_phases_s", "h2d_gb_per_step", "adam_busy_s_per_step",
                                 "fetch_blocked_on_adam_s_per_step", "comm", "losses", "losses_finite",
                                 "traced_step", "per_rank", "attn_implementation") if k in res}
    line["detail"] = extra
    return line


if __name__ == "__main__":
    main()
