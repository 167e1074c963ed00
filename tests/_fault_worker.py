"""Workers for host-side fault tests (CPU / gloo): one rank stops between
steps; the survivor must fail with a bounded, descriptive error."""
import os
import sys
import time
import traceback

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def run(rank, world, port, out_path, grad_mode):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_RANK=str(rank),
                      LOCAL_WORLD_SIZE=str(world), T1_QUIET="1")
    result = {"rank": rank, "error": None, "steps": 0}
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        cfg = LlamaConfig.tiny()
        torch.manual_seed(0)
        eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(
            dtype=torch.float32, device="cpu", grad_sync_mode=grad_mode, host_wait_timeout_s=3.0))
        ids = torch.randint(0, cfg.vocab_size, (1, 32))
        for step in range(3):
            if rank == 1 and step == 1:
                # this rank leaves between steps: nothing of it is in flight
                result["left"] = True
                torch.save(result, out_path + f".{rank}")
                os._exit(0)
            eng(input_ids=ids, labels=ids)
            result["steps"] += 1
        eng.wait_for_updates()
    except Exception as exc:  # the survivor lands here
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()
    torch.save(result, out_path + f".{rank}")
    os._exit(0)


def run_mismatch(rank, world, port, out_path):
    """Rank 1 builds a model with one layer fewer than rank 0's: it must
    refuse the shared region rank 0 laid out instead of reading it."""
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_RANK=str(rank),
                      LOCAL_WORLD_SIZE=str(world), T1_QUIET="1")
    result = {"rank": rank, "error": None}
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        cfg = LlamaConfig.tiny()
        if rank == 1:
            cfg.num_hidden_layers -= 1
        eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.float32, device="cpu",
                                                               host_wait_timeout_s=3.0))
        eng.close()
    except Exception as exc:
        result["error"] = f"{type(exc).__name__}: {exc}"
    torch.save(result, out_path + f".{rank}")
    os._exit(0)


def run_multinode(rank, world, port, out_path):
    """Two ranks that claim to sit on different nodes (one local rank
    each): both must refuse with a named error."""
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_RANK="0",
                      LOCAL_WORLD_SIZE="1", T1_QUIET="1")
    result = {"rank": rank, "error": None}
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        SlideFSDP(LlamaForCausalLM(LlamaConfig.tiny()), SlideFSDPConfig(dtype=torch.float32, device="cpu"))
    except Exception as exc:
        result["error"] = f"{type(exc).__name__}: {exc}"
    torch.save(result, out_path + f".{rank}")
    os._exit(0)
