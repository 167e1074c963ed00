"""Worker for multi-rank CPU (gloo) engine tests; imported by tests."""
import os
import sys
import traceback

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def batches(cfg, world, steps, batch=2, seq=32):
    g = torch.Generator().manual_seed(123)
    return [[torch.randint(0, cfg.vocab_size, (batch, seq), generator=g) for _ in range(world)]
            for _ in range(steps)]


def run_engine(rank, world, port, mode, grad, sharding, steps, out_path, ckpt, extra=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["LOCAL_WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["T1_QUIET"] = "1"
    try:
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        cfg = LlamaConfig.tiny()
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg)
        conf = SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3, weight_decay=0.01,
                               param_transfer_mode=mode, grad_sync_mode=grad,
                               optimizer_sharding=sharding, enable_activation_checkpoint=ckpt,
                               **(extra or {}))
        eng = SlideFSDP(model, conf)
        # the shared-memory file is gone once every rank has mapped it
        assert eng.shared.shm_path is None or not os.path.exists(eng.shared.shm_path)
        losses = []
        for step_batches in batches(cfg, world, steps):
            ids = step_batches[rank]
            losses.append(float(eng(input_ids=ids, labels=ids).loss))
        eng.wait_for_updates()
        dist.barrier()
        if rank == 0:
            master = {n: t.clone() for n, t in eng.named_master_tensors()}
            torch.save({"losses": losses, "master": master, "grad_norm": eng.last_grad_norm}, out_path)
        else:
            torch.save({"losses": losses}, out_path + f".{rank}")
        dist.barrier()
        eng.close()
        dist.destroy_process_group()
    except Exception:
        with open(out_path + f".err{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise


def run_state(rank, world, port, sharding, load_dir, save_dir, steps, err_path):
    """Optionally load a saved state, train ``steps`` steps (2 x 32 tokens
    per rank), then save the state."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["LOCAL_WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["T1_QUIET"] = "1"
    try:
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        cfg = LlamaConfig.tiny()
        torch.manual_seed(0)
        eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3,
                                                               optimizer_sharding=sharding))
        if load_dir:
            eng.load_state(load_dir)
        for step_batches in batches(cfg, world, steps):
            ids = step_batches[rank]
            eng(input_ids=ids, labels=ids)
        eng.save_state(save_dir)
        eng.close()
        dist.destroy_process_group()
    except Exception:
        with open(err_path + f".err{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise
