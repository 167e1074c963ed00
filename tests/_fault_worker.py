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


def run(rank, world, port, out_path, grad_mode, leave="exit", gpu=False):
    """Rank 1 trains one step and leaves: ``leave="exit"`` stops the
    process (as a crash would), ``"close"`` closes its engine first.  The
    survivor's next step must fail on the host with an error naming rank 1.
    ``gpu``: NCCL ranks on cuda:<rank> with NVLS off and NCCL collectives
    only (no symmetric memory), short process-group timeout."""
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_RANK=str(rank),
                      LOCAL_WORLD_SIZE=str(world), T1_QUIET="1")
    if gpu:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
    result = {"rank": rank, "error": None, "steps": 0}
    try:
        if gpu:
            torch.cuda.set_device(rank)
            dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=20),
                                    device_id=torch.device("cuda", rank))
        else:
            dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        torch.manual_seed(0)
        if gpu:
            cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                              num_attention_heads=4, num_key_value_heads=2)
            conf = SlideFSDPConfig(dtype=torch.bfloat16, device=torch.device("cuda", rank),
                                   grad_sync_mode=grad_mode, fused_comm=False, host_wait_timeout_s=5.0)
            ids = torch.randint(0, cfg.vocab_size, (2, 128)).cuda()
        else:
            cfg = LlamaConfig.tiny()
            conf = SlideFSDPConfig(dtype=torch.float32, device="cpu", grad_sync_mode=grad_mode,
                                   host_wait_timeout_s=3.0)
            ids = torch.randint(0, cfg.vocab_size, (1, 32))
        eng = SlideFSDP(LlamaForCausalLM(cfg, device="meta" if gpu else None), conf)
        for step in range(3):
            if rank == 1 and step == 1:
                # this rank leaves between steps: nothing of it is in flight
                if leave == "close":
                    eng.close()
                if gpu:
                    torch.cuda.synchronize()
                result["left"] = True
                torch.save(result, out_path + f".{rank}")
                os._exit(0)
            eng(input_ids=ids, labels=ids)
            result["steps"] += 1
            if gpu:
                eng.wait_for_updates()
                torch.cuda.synchronize()
        eng.wait_for_updates()
    except Exception as exc:  # the survivor lands here
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()
        result["t_error"] = time.time()
    if gpu:
        # the survivor's GPU still answers: a kernel runs and nothing is sticky
        try:
            x = torch.ones(1 << 20, device=torch.device("cuda", rank))
            result["gpu_ok"] = float(x.sum().item()) == float(1 << 20)
            torch.cuda.synchronize()
        except Exception as exc:
            result["gpu_ok"] = False
            result["gpu_error"] = repr(exc)
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
