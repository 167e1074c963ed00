"""FSDP arm of bench.py (``--impl fsdp``): the reference's PyTorch-FSDP
comparison script (baseline/fsdp_baseline.py in the reference tree, copied
verbatim into baseline/_ref) driven through its own functions:

    TrainConfig(...)  setup_fsdp(model, cfg, device)  prepare_optimizer(model, cfg)

with the settings of its fsdp_config.json (full_shard, CPU offload of
parameters, backward_pre prefetch, forward prefetch, limit_all_gathers,
transformer auto-wrap, bf16 mixed precision with bf16 reduction, grad-norm
clipping 1.0) and one training step exactly as its ``train_one_epoch`` runs
it: forward, ``loss.backward()``, ``clip_grad_norm_``, ``optimizer.step()``,
``zero_grad``.  The model is the same random-init Llama-3.1-8B-architecture
HF model the reference arm uses, in bf16 on the CPU (what the script's
``get_model`` loads); batches are synthetic tokens of this bench's shape.
Timing is on the device (CUDA events), max over ranks."""
from __future__ import annotations

import os
import sys
import time

from baseline.reference_arm import REF, build_hf_model


def run(args, rank, world, local):
    import torch
    import torch.distributed as dist

    path = os.path.join(REF, "baseline", "fsdp_baseline.py")
    if not os.path.exists(path):
        return {"unavailable": "reference FSDP baseline not present in baseline/_ref"}
    if world == 1 and not dist.is_initialized():
        # FSDP needs a process group even on one GPU
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", local))
    sys.path.insert(0, REF)
    sys.path.insert(0, os.path.join(REF, "baseline"))
    try:
        import fsdp_baseline as fb  # the reference's own script
    except Exception as exc:  # pragma: no cover - depends on the box
        return {"unavailable": f"reference FSDP baseline import failed: {type(exc).__name__}: {exc}"}

    dev = torch.device("cuda", local)
    t0 = time.time()
    model, attn = build_hf_model(args.model, dev, tuple_layers=False)
    cfg = fb.TrainConfig(max_seq_length=args.seq, train_batch_size=args.batch, learning_rate=1e-5,
                         weight_decay=0.01, dtype="bf16", attention_implementation=attn,
                         sharding_strategy="full_shard", cpu_offload=True, backward_prefetch="backward_pre",
                         forward_prefetch=True, limit_all_gathers=True, wrap_policy="transformer",
                         mixed_precision_reduce_dtype="bf16", clip_grad_norm=1.0)
    fb.set_seed(cfg.seed + rank)
    fsdp_model = fb.setup_fsdp(model, cfg, dev)
    optimizer = fb.prepare_optimizer(fsdp_model, cfg)
    init_s = time.time() - t0

    V = model.config.vocab_size
    g = torch.Generator().manual_seed(1000 + rank)
    n = args.warmup + 2 * args.steps
    batches = [torch.randint(0, V, (args.batch, args.seq), generator=g).pin_memory() for _ in range(n)]
    dev_batches = [b.to(dev) for b in batches]

    def step(ids):
        out = fsdp_model(input_ids=ids, labels=ids)
        loss = out.loss
        loss.backward()
        if cfg.clip_grad_norm > 0:
            fsdp_model.clip_grad_norm_(cfg.clip_grad_norm)
        optimizer.step()
        optimizer.zero_grad(set_to_none=True)
        return loss

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    losses = []
    fsdp_model.train()
    for i in range(args.warmup):
        losses.append(float(step(dev_batches[i]).detach()))
    barrier()

    from bench import ClockSampler, max_over_ranks

    sampler = ClockSampler(local)
    sampler.start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier()
    start.record()
    last = None
    for k in range(args.steps):
        last = step(dev_batches[args.warmup + k])
    end.record()
    end.synchronize()
    barrier()
    clocks = sampler.stop()
    dev_ms = max_over_ranks(start.elapsed_time(end), world)
    losses.append(float(last.detach()))

    e2e = None
    if not args.no_e2e:
        barrier()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record()
        for k in range(args.steps):
            ids = batches[args.warmup + args.steps + k].to(dev, non_blocking=True)
            losses.append(step(ids).item())
        e_end.record()
        e_end.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
        tokens = args.batch * args.seq * world * args.steps
        e2e = {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": "tokens/s",
               "h2d_bytes_per_step": int(args.batch * args.seq * 8), "d2h_bytes_per_step": 4}
    return {"dev_ms": dev_ms, "e2e": e2e, "clocks": clocks, "launches": 0, "init_s": init_s,
            "losses": losses, "attn_implementation": attn}
