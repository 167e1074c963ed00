"""Training CLI (same flags as the reference's train.py, train.py:228-314).

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 train.py --model-path /path/to/hf_llama
    torchrun ... train.py --model-config llama31_8b        # random init, no checkpoint needed
    torchrun ... train.py --config train_config.json --param-transfer-mode shard

`--model-path` loads an HF-layout Llama checkpoint directory (config.json +
safetensors); `--model-config` builds a random-init model from a preset
(llama31_8b, llama_70b, tiny).  Data is the synthetic DummyDataset (random
tokens, right padding, -100 on padding and an instruction prefix).  Loss,
tokens/s (device-timed per logging window) and TFLOPS are printed by rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="test1_b200 layer-sliding training",
                                formatter_class=argparse.ArgumentDefaultsHelpFormatter)
    p.add_argument("--config", type=str, default=None, help="JSON config file (SlideFSDPConfig fields)")
    p.add_argument("--model-path", type=str, default=None, help="HF-layout Llama checkpoint directory")
    p.add_argument("--model-config", type=str, default=None, help="random-init preset: llama31_8b | llama_70b | tiny")
    p.add_argument("--param-transfer-mode", type=str, choices=["full", "shard"], default=None)
    p.add_argument("--grad-sync-mode", type=str, choices=["gpu_reduce", "cpu_reduce"], default=None)
    p.add_argument("--batch-size", type=int, default=None, help="per-GPU batch size")
    p.add_argument("--seq-length", type=int, default=None)
    p.add_argument("--num-epochs", type=int, default=None)
    p.add_argument("--max-steps", type=int, default=0, help="stop after this many steps (0 = full epochs)")
    p.add_argument("--lr", type=float, default=None)
    p.add_argument("--output-dir", type=str, default="./output")
    p.add_argument("--save-model", action="store_true")
    p.add_argument("--save-state", action="store_true", help="also save master + optimizer state")
    p.add_argument("--plan", action="store_true",
                   help="print the host and device memory this run needs (GB) and exit")
    p.add_argument("--lr-scheduler", choices=["constant", "linear", "cosine"], default="constant",
                   help="per-step learning-rate schedule after --warmup-steps of linear warm-up")
    p.add_argument("--warmup-steps", type=int, default=0)
    p.add_argument("--save-state-every", type=int, default=0,
                   help="also save master + optimizer state every N steps (output_dir/state_step<N>; "
                        "the two newest are kept, output_dir/latest_state names the newest)")
    p.add_argument("--resume", type=str, default=None,
                   help="directory written by --save-state / --save-state-every, or an output_dir "
                        "holding latest_state (the world size may differ from the saving run's)")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--device", type=str, default=None, help="override device (e.g. cpu)")
    return p.parse_args(argv)


def load_config(args):
    from test1_b200 import SlideFSDPConfig

    d = {}
    if args.config:
        with open(args.config, "r", encoding="utf-8") as f:
            d = json.load(f)
    for flag, key in [("model_path", "model_path"), ("param_transfer_mode", "param_transfer_mode"),
                      ("grad_sync_mode", "grad_sync_mode"), ("batch_size", "train_batch_size"),
                      ("seq_length", "max_seq_length"), ("num_epochs", "num_epochs"), ("lr", "lr"),
                      ("seed", "seed"), ("device", "device")]:
        v = getattr(args, flag)
        if v is not None:
            d[key] = v
    return SlideFSDPConfig.from_dict(d)


def init_distributed(device_type: str):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if device_type == "cuda":
        torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl" if device_type == "cuda" else "gloo",
                                timeout=timedelta(seconds=900))
    pin_main_thread(rank)
    return rank, world, local


def pin_main_thread(rank: int) -> None:
    """Pin the launching thread to the control cores numa_launch.sh chose
    (NUMA_CONTROL_CORES, a CPU list such as "0-1,8"), as the reference's
    train.py does; the host worker pool pins its own threads to
    NUMA_CPU_ADAM_CORES."""
    spec = os.environ.get("NUMA_CONTROL_CORES", "").strip()
    if not spec:
        return
    cpus = []
    for part in spec.split(","):
        part = part.strip()
        if "-" in part:
            a, b = part.split("-", 1)
            cpus.extend(range(int(a), int(b) + 1))
        elif part:
            cpus.append(int(part))
    try:
        os.sched_setaffinity(0, cpus)
    except OSError as exc:
        print(f"[rank {rank}] could not pin the main thread to {spec}: {exc}", flush=True)


def build_model(args, config):
    from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
    from test1_b200.utils.checkpoint_io import load_hf_checkpoint

    if args.model_path or config.model_path:
        path = args.model_path or config.model_path
        hf_cfg, tensors = load_hf_checkpoint(path)
        d = hf_cfg if isinstance(hf_cfg, dict) else hf_cfg.to_dict()
        llama_like = (d.get("model_type") in ("llama", "mistral") and not d.get("attention_bias")
                      and not d.get("mlp_bias") and not d.get("tie_word_embeddings"))
        if not llama_like:
            # any other HF causal LM: its own modules, run by the engine's
            # generic layer path (the reference loads with AutoModelForCausalLM)
            import torch
            from transformers import AutoModelForCausalLM

            return AutoModelForCausalLM.from_pretrained(path, dtype=torch.float32)
        cfg = LlamaConfig.from_hf(hf_cfg)
        model = LlamaForCausalLM(cfg, device="meta")
        for name, p in model.named_parameters():
            if name not in tensors:
                raise ValueError(f"checkpoint lacks {name}")
            p.data = tensors[name].float()
        return model
    preset = args.model_config or "tiny"
    return LlamaForCausalLM(getattr(LlamaConfig, preset)(), device="meta")


def main(argv=None):
    args = parse_args(argv)
    import torch

    from test1_b200.slide_fsdp import SlideFSDP
    from test1_b200.utils.datasets import DummyDataset
    from test1_b200.utils.metric import calculate_flops_per_batch

    config = load_config(args)
    rank, world, local = init_distributed(config.device.type)
    if config.device.type == "cuda":
        config.device = torch.device("cuda", local)
    random.seed(config.seed + rank)
    torch.manual_seed(config.seed + rank)

    model = build_model(args, config)
    mcfg = model.config
    if args.plan:
        from test1_b200.utils.memory_plan import plan_memory

        if not hasattr(mcfg, "decoder_layer_params"):
            raise SystemExit("--plan needs a Llama-structured model")
        if rank == 0:
            plan = plan_memory(mcfg, config, world, config.train_batch_size, config.max_seq_length)
            print(json.dumps({k: round(v, 3) for k, v in plan.items()}), flush=True)
        return
    flops = calculate_flops_per_batch(mcfg, config.train_batch_size, config.max_seq_length) * world
    engine = SlideFSDP(model, config)
    if args.resume:
        src = args.resume
        marker = os.path.join(src, "latest_state")
        if os.path.isfile(marker):
            with open(marker) as f:
                src = os.path.join(src, f.read().strip())
        engine.load_state(src)
        if rank == 0:
            print(f"Resumed from {src}", flush=True)

    from torch.utils.data import DataLoader
    from torch.utils.data.distributed import DistributedSampler

    ds = DummyDataset(size=1024 * config.num_epochs, max_length=config.max_seq_length,
                      vocab_size=mcfg.vocab_size, seed=config.seed)
    sampler = DistributedSampler(ds, num_replicas=world, rank=rank, shuffle=True) if world > 1 else None
    loader = DataLoader(ds, batch_size=config.train_batch_size, sampler=sampler,
                        shuffle=sampler is None, drop_last=True, pin_memory=config.device.type == "cuda")
    tokens_per_step = config.train_batch_size * config.max_seq_length * world
    total_steps = len(loader) * config.num_epochs
    if args.max_steps:
        total_steps = min(total_steps, args.max_steps)
    base_lr = config.lr
    step = 0
    timed = config.device.type == "cuda"
    for epoch in range(1, config.num_epochs + 1):
        if sampler is not None:
            sampler.set_epoch(epoch)
        t_start = time.perf_counter()
        ev0 = torch.cuda.Event(enable_timing=True) if timed else None
        if timed:
            ev0.record()
        running = 0.0
        for batch in loader:
            if args.lr_scheduler != "constant" or args.warmup_steps:
                engine.update_learning_rate(
                    scheduled_lr(base_lr, step, total_steps, args.warmup_steps, args.lr_scheduler))
            batch = {k: v.to(config.device, non_blocking=True) for k, v in batch.items()}
            out = engine(input_ids=batch["input_ids"], attention_mask=batch["attention_mask"],
                         labels=batch["labels"])
            step += 1
            running += float(out.loss)
            if step % max(1, config.log_every_n_steps) == 0:
                if timed:
                    ev1 = torch.cuda.Event(enable_timing=True)
                    ev1.record()
                    ev1.synchronize()
                    dt = ev0.elapsed_time(ev1) / 1e3
                    ev0 = ev1
                else:
                    dt = time.perf_counter() - t_start
                    t_start = time.perf_counter()
                n = max(1, config.log_every_n_steps)
                if rank == 0:
                    gn = getattr(engine, "last_grad_norm", None)
                    gn = f" | grad norm {gn:.4f}" if gn is not None else ""
                    print(f"Epoch {epoch} | Step {step} | Loss: {running / n:.4f} | "
                          f"{tokens_per_step * n / dt:.1f} tokens/s | {flops * n / dt / 1e12:.2f} TFLOPS | "
                          f"lr {engine.config.lr:.3g}{gn}",
                          flush=True)
                running = 0.0
            if args.save_state_every and step % args.save_state_every == 0:
                save_periodic_state(engine, args.output_dir, step, rank, world)
            if args.max_steps and step >= args.max_steps:
                break
        if args.max_steps and step >= args.max_steps:
            break
    engine.wait_for_updates()
    if args.save_model:
        engine.save_pretrained(args.output_dir)
    if args.save_state:
        engine.save_state(os.path.join(args.output_dir, "state"))
    engine.close()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print("Training completed!")


def scheduled_lr(base: float, step: int, total: int, warmup: int, kind: str) -> float:
    """Learning rate of step ``step`` (0-based): linear warm-up over
    ``warmup`` steps, then constant, linear decay to 0, or half-cosine decay
    to 0 at ``total`` steps."""
    if warmup and step < warmup:
        return base * (step + 1) / warmup
    if kind == "constant" or total <= warmup:
        return base
    frac = min(1.0, (step - warmup) / max(1, total - warmup))
    if kind == "linear":
        return base * (1.0 - frac)
    return base * 0.5 * (1.0 + math.cos(math.pi * frac))


def save_periodic_state(engine, output_dir: str, step: int, rank: int, world: int) -> None:
    """Save the full training state into output_dir/state_step<step>; once
    every rank has written its part, rank 0 points latest_state at it and
    drops all but the two newest such directories, so a crash during a save
    always leaves a complete earlier one."""
    import shutil

    name = f"state_step{step}"
    engine.save_state(os.path.join(output_dir, name))  # ends with a barrier on every rank
    if rank == 0:
        tmp = os.path.join(output_dir, "latest_state.tmp")
        with open(tmp, "w") as f:
            f.write(name)
        os.replace(tmp, os.path.join(output_dir, "latest_state"))
        old = sorted((d for d in os.listdir(output_dir) if d.startswith("state_step") and d[10:].isdigit()),
                     key=lambda d: int(d[10:]))
        for d in old[:-2]:
            shutil.rmtree(os.path.join(output_dir, d), ignore_errors=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


if __name__ == "__main__":
    main()
