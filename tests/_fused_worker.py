"""Worker processes for the 2-GPU fused-communication tests."""
import os
import sys
import traceback

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _init(rank, world, port):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_RANK=str(rank),
                      LOCAL_WORLD_SIZE=str(world), RANK=str(rank), WORLD_SIZE=str(world),
                      T1_QUIET="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def kernels(rank, world, port, out_path):
    try:
        _init(rank, world, port)
        from test1_b200 import _native
        from test1_b200.parallel.fused import SymmetricBuffer
        from test1_b200.runtime.layer_state import shard_bounds

        C = _native.cuda()
        dev = torch.device("cuda", rank)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        P = 1000 * 64 + 24
        buf = SymmetricBuffer(P, torch.bfloat16, dev, dist.group.WORLD)
        pbuf = SymmetricBuffer(P, torch.bfloat16, dev, dist.group.WORLD)
        s, e = shard_bounds(P, world, rank)
        ok = True
        msgs = []
        for it in range(3):
            g = torch.Generator(device=dev).manual_seed(100 * it + rank)
            vals = torch.randn(P, device=dev, generator=g).bfloat16()
            buf.tensor.copy_(vals)
            torch.cuda.synchronize()
            dist.barrier()
            out = torch.empty(max(e - s, 1), dtype=torch.bfloat16, pin_memory=True)
            C.fused_rs_d2h(buf.ptrs, buf.sigs, rank, world, s, e - s, out, 1.0 / world,
                           buf.next_epoch(), buf.counter, err)
            torch.cuda.synchronize()
            allv = [torch.empty_like(vals) for _ in range(world)]
            dist.all_gather(allv, vals)
            expect = (sum(v.float() for v in allv) / world)[s:e].bfloat16().cpu()
            diff = (out[: e - s].float() - expect.float()).abs().max().item()
            if diff > 1e-2:
                ok = False
                msgs.append(f"rs it{it} diff {diff}")
            # shard gather from an fp32 host master
            master = torch.randn(P, generator=torch.Generator().manual_seed(7 + it)).pin_memory()
            pbuf.tensor.zero_()
            torch.cuda.synchronize()
            dist.barrier()
            C.fused_shard_gather(pbuf.ptrs, pbuf.sigs, rank, world, s, e - s, master[s:e], None,
                                 pbuf.next_epoch(), pbuf.counter, err)
            torch.cuda.synchronize()
            if not torch.equal(pbuf.tensor.cpu(), master.bfloat16()):
                ok = False
                msgs.append(f"gather(fp32) it{it} mismatch")
            # split master: both planes, rebuilt and rounded on the GPU
            hi = torch.empty(P, dtype=torch.bfloat16).pin_memory()
            lo = torch.empty(P, dtype=torch.int16).pin_memory()
            _native.host().f32_to_split(master, hi, lo)
            pbuf.tensor.zero_()
            torch.cuda.synchronize()
            dist.barrier()
            C.fused_shard_gather(pbuf.ptrs, pbuf.sigs, rank, world, s, e - s, hi[s:e], lo[s:e],
                                 pbuf.next_epoch(), pbuf.counter, err)
            torch.cuda.synchronize()
            if not torch.equal(pbuf.tensor.cpu(), master.bfloat16()):
                ok = False
                msgs.append(f"gather it{it} mismatch")
            # staged: this rank's shard already in its own unit (copy
            # engine), the kernel only broadcasts it, on a capped grid
            pbuf.tensor.zero_()
            torch.cuda.synchronize()
            dist.barrier()
            pbuf.tensor[s:e].copy_(master.bfloat16()[s:e], non_blocking=True)
            C.fused_shard_gather(pbuf.ptrs, pbuf.sigs, rank, world, s, e - s, pbuf.tensor[s:e], None,
                                 pbuf.next_epoch(), pbuf.counter, err, 4)
            torch.cuda.synchronize()
            if not torch.equal(pbuf.tensor.cpu(), master.bfloat16()):
                ok = False
                msgs.append(f"staged gather it{it} mismatch")
        if int(err.item()) != 0:
            ok = False
            msgs.append(f"err {int(err.item())}")
        torch.save({"ok": ok, "msgs": msgs}, out_path + f".{rank}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(out_path + f".err{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise


def engine(rank, world, port, out_path, mode, fused, extra=None):
    try:
        _init(rank, world, port)
        from test1_b200 import SlideFSDPConfig
        from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
        from test1_b200.slide_fsdp import SlideFSDP

        cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                          num_attention_heads=4, num_key_value_heads=2)
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg)
        eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.bfloat16, device=torch.device("cuda", rank),
                                               lr=1e-3, param_transfer_mode=mode,
                                               grad_sync_mode="gpu_reduce", fused_comm=fused,
                                               **(extra or {})))
        g = torch.Generator().manual_seed(11)
        losses = []
        for step in range(3):
            batch = [torch.randint(0, cfg.vocab_size, (2, 128), generator=g) for _ in range(world)]
            ids = batch[rank].cuda()
            losses.append(float(eng(input_ids=ids, labels=ids).loss))
        eng.wait_for_updates()
        res = {"losses": losses, "comm": eng.comm.name}
        if rank == 0:
            res["master"] = {n: t.clone() for n, t in eng.named_master_tensors()}
        torch.save(res, out_path + f".{rank}")
        dist.barrier()
        eng.close()
        dist.destroy_process_group()
    except Exception:
        with open(out_path + f".err{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise


def ag_gemm(rank, world, port, out_path, src_kind):
    """fused_ag_qkv: gather a layer (fp32 master shards on the host) into every
    rank's unit and compute x @ W_qkv^T from it; compare with a plain GEMM on
    the gathered weights."""
    try:
        _init(rank, world, port)
        from test1_b200 import _native
        from test1_b200.ops import native
        from test1_b200.parallel.fused import SymmetricBuffer
        from test1_b200.runtime.layer_state import shard_bounds

        C = _native.cuda()
        dev = torch.device("cuda", rank)
        K, n_rows, T = 512, 768, 384
        P = n_rows * K + 100 * 1024 + 8      # weight rows followed by other params
        unit = SymmetricBuffer(P, torch.bfloat16, dev, dist.group.WORLD)
        counters = torch.zeros(65, dtype=torch.int32, device=dev)
        shards = torch.tensor([list(shard_bounds(P, world, q)) for q in range(world)], dtype=torch.int64)
        s, e = shard_bounds(P, world, rank)
        ok, msgs = True, []
        for it in range(3):
            master = torch.randn(P, generator=torch.Generator().manual_seed(31 + it)) * 0.05
            lo = None
            if src_kind == "staged":
                src = unit.tensor[s:e]  # filled below, after the zero fill
            elif src_kind == "split":
                hi_all = torch.empty(P, dtype=torch.bfloat16)
                lo_all = torch.empty(P, dtype=torch.int16)
                _native.host().f32_to_split(master, hi_all, lo_all)
                src = hi_all[s:e].contiguous().pin_memory()
                lo = lo_all[s:e].contiguous().pin_memory()
            else:
                src = (master if src_kind == "fp32" else master.bfloat16())[s:e].contiguous().pin_memory()
            x = torch.randn(T, K, generator=torch.Generator().manual_seed(77 + it)).bfloat16().to(dev)
            out = torch.empty(T, n_rows, dtype=torch.bfloat16, device=dev)
            unit.tensor.zero_()
            if src_kind == "staged":
                unit.tensor[s:e].copy_(master.bfloat16()[s:e])
            torch.cuda.synchronize()
            dist.barrier()
            C.fused_ag_qkv(x, unit.tensor, n_rows, out, unit.ptrs, unit.sigs, shards, rank, world,
                           src, lo, unit.next_epoch(), counters)
            torch.cuda.synchronize()
            full = master.bfloat16().to(dev)
            if not torch.equal(unit.tensor, full):
                ok = False
                msgs.append(f"it{it}: gathered layer differs")
            ref = x.float() @ full[: n_rows * K].view(n_rows, K).float().t()
            rel = ((out.float() - ref).norm() / ref.norm()).item()
            if rel > 6e-3:
                ok = False
                msgs.append(f"it{it}: gemm rel err {rel}")
        code = native.gemm_error()
        if code:
            ok = False
            msgs.append(f"gemm error word {code}")
        torch.save({"ok": ok, "msgs": msgs}, out_path + f".{rank}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(out_path + f".err{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise
