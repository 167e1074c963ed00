"""Comparison config 1: the tiny Llama-style decoder trained on CPU ranks over
gloo (world size 2, param_transfer_mode=full, grad_sync_mode=cpu_reduce, fp32
throughout, LayerAdam in AdamW mode, lr 1e-5, 10 steps), checked step by step
against a single-process oracle: HF ``LlamaForCausalLM`` with the same
weights whose per-step gradient is the mean of the two ranks' gradients,
stepped by ``torch.optim.AdamW``.

Architecture: 4 layers, hidden 256, 4 heads (dim 64), 2 KV heads, SwiGLU 688,
vocab 1024, RoPE theta 10000, RMSNorm eps 1e-5, untied embeddings; weights
N(0, 0.02) from seed 0.  Rank r draws its batch (2 x 128 tokens uniform in
[0, 1024)) from a generator seeded 1 + r; labels are the inputs (the loss
shifts them by one).  The reference cannot run this configuration: its
activation checkpointing allocates a CUDA stream at import
(sliding_checkpoint.py:8).

    python benchmark/plumbing_cpu.py [--steps 10] [--world 2] [--grad-sync cpu_reduce]

Prints one JSON line: per-step losses of both sides, the largest loss and
parameter differences, and the engine's wall time per step (CPU).
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import sys
import tempfile
import time
import traceback

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

BATCH, SEQ, LR, WD = 2, 128, 1e-5, 0.01


def _batches(vocab, rank, steps):
    g = torch.Generator().manual_seed(1 + rank)
    return [torch.randint(0, vocab, (BATCH, SEQ), generator=g) for _ in range(steps)]


def build_model():
    """The config-1 model with weights N(0, 0.02) from seed 0 (norms 1)."""
    from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig.tiny()
    model = LlamaForCausalLM(cfg, device="meta")
    model = model.to_empty(device="cpu")
    model.init_weights(seed=0)
    return model


def _rank_main(rank, world, port, steps, grad_sync, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), T1_QUIET="1")
    try:
        from datetime import timedelta

        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.slide_fsdp import SlideFSDP

        model = build_model()
        conf = SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=LR, weight_decay=WD,
                               param_transfer_mode="full", grad_sync_mode=grad_sync)
        eng = SlideFSDP(model, conf)
        losses, times = [], []
        for ids in _batches(model.config.vocab_size, rank, steps):
            t0 = time.perf_counter()
            losses.append(float(eng(input_ids=ids, labels=ids).loss))
            times.append(time.perf_counter() - t0)
        eng.wait_for_updates()
        dist.barrier()
        res = {"losses": losses, "times": times}
        if rank == 0:
            res["master"] = {n: t.clone() for n, t in eng.named_master_tensors()}
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
        eng.close()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise


def oracle(world, steps):
    """Per-rank losses and final parameters of HF Llama + torch AdamW with the
    ranks' mean gradient."""
    import transformers

    model = build_model()
    hf = transformers.LlamaForCausalLM(model.config.to_hf()).float()
    hf.config._attn_implementation = "eager"
    hf.load_state_dict({n: p.detach().clone() for n, p in model.named_parameters()})
    opt = torch.optim.AdamW(hf.parameters(), lr=LR, betas=(0.9, 0.999), eps=1e-8, weight_decay=WD)
    per_rank = [_batches(model.config.vocab_size, r, steps) for r in range(world)]
    losses = [[] for _ in range(world)]
    for s in range(steps):
        opt.zero_grad()
        for r in range(world):
            ids = per_rank[r][s]
            loss = hf(input_ids=ids, labels=ids).loss
            (loss / world).backward()
            losses[r].append(float(loss.detach()))
        opt.step()
    return losses, {n: p.detach() for n, p in hf.named_parameters()}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def run(steps=10, world=2, grad_sync="cpu_reduce"):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as out_dir:
        port = _free_port()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, steps, grad_sync, out_dir))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
        errs = sorted(f for f in os.listdir(out_dir) if f.endswith(".err"))
        if errs:
            raise RuntimeError(open(os.path.join(out_dir, errs[0])).read())
        if any(p.exitcode != 0 for p in procs):
            raise RuntimeError(f"rank exit codes {[p.exitcode for p in procs]}")
        res = [torch.load(os.path.join(out_dir, f"rank{r}.pt")) for r in range(world)]
    want_losses, want_params = oracle(world, steps)
    loss_diff = max(abs(res[r]["losses"][s] - want_losses[r][s]) for r in range(world) for s in range(steps))
    param_diff = max((res[0]["master"][n].view(p.shape) - p).abs().max().item() for n, p in want_params.items())
    # the first step includes lazy setup; report the steady-state steps
    per_step = [max(res[r]["times"][s] for r in range(world)) for s in range(steps)]
    steady = per_step[1:] or per_step
    return {
        "config": {"model": "tiny Llama (4 x 256, GQA 4/2, SwiGLU 688, vocab 1024)", "world_size": world,
                   "backend": "gloo", "param_transfer_mode": "full", "grad_sync_mode": grad_sync,
                   "dtype": "fp32", "batch_per_rank": BATCH, "seq_len": SEQ, "lr": LR, "steps": steps},
        "losses": [res[r]["losses"] for r in range(world)],
        "oracle_losses": want_losses,
        "max_loss_diff": loss_diff,
        "max_param_diff": param_diff,
        "ms_per_step": 1000.0 * sum(steady) / len(steady),
        "tokens_per_s": world * BATCH * SEQ * len(steady) / sum(steady),
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--grad-sync", default="cpu_reduce", choices=["cpu_reduce", "gpu_reduce"])
    a = ap.parse_args()
    print(json.dumps(run(a.steps, a.world, a.grad_sync)))


if __name__ == "__main__":
    main()
