"""Reference arm of bench.py: the unmodified SlideFSDP reference (source tree
copied verbatim into baseline/_ref, since it ships no packaging metadata and
`pip install` refuses it) driven through its own public API:

    from config import SlideFSDPConfig; from slide_fsdp import SlideFSDP
    model = SlideFSDP(hf_llama, SlideFSDPConfig(...)); out = model(input_ids=..., labels=...)

What this harness provides around it (none of it touches the reference's
code path):
  * an HF transformers LlamaForCausalLM of the Llama-3.1-8B architecture,
    random N(0, 0.02) weights in bf16 on the CPU (what the reference's
    train.py loads with `from_pretrained(device_map="cpu", torch_dtype=bf16)`),
    with Liger's Llama patches applied as `AutoLigerKernelForCausalLM` does;
  * the decoder layers return a 1-tuple, the contract of transformers 4.x
    that the reference indexes with `[0]` (slide_fsdp.py:590); the installed
    transformers 5.x returns a bare tensor;
  * OMP threads as the reference's numa_launch.sh assigns them (rank 0 gets
    the spare cores, the other ranks one control core each);
  * the random weights are drawn on the CPU, so, as under the reference's own
    train.py (`from_pretrained(device_map="cpu")`), the GPU holds nothing
    before SlideFSDP allocates its pool.  This matters: the reference's last
    decoder layer stays resident between its forward and backward, so its
    backward fetch returns early (layer_state.py:285-287) without zeroing the
    pool unit's gradient buffer or pointing `param.grad` at it; the gradient
    copy to the host (layer_state.py:367-381) then reads a buffer the backward
    never wrote, and LayerAdam applies it (layer_adam.py:404-417).  On fresh
    device memory that buffer holds zeros (step 1) or stale gradients of other
    layers (later steps), so losses stay finite; after a GPU-side random
    initialisation it held fp32 random bits whose low halves include bf16
    NaN/Inf patterns, and every loss after the first update was NaN;
  * the same synthetic batches, timing and JSON fields as our own arm.
"""
from __future__ import annotations

import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def omp_threads_for_rank(local_rank: int, local_world: int, ncpu: int) -> int:
    """numa_launch.sh policy on a single NUMA node: one control core per
    rank; rank 0 also owns every spare core for its CPU Adam."""
    if local_world <= 1:
        return ncpu
    return max(1, ncpu - local_world) if local_rank == 0 else 1


def _tuple_layers(model):
    import torch.nn as nn

    class TupleOut(nn.Module):
        def __init__(self, inner):
            super().__init__()
            self.inner = inner

        def forward(self, *args, **kwargs):
            out = self.inner(*args, **kwargs)
            return out if isinstance(out, tuple) else (out,)

    dec = model.get_decoder()
    dec.layers = nn.ModuleList(TupleOut(l) for l in dec.layers)
    return model


def build_hf_model(model_name: str, device_for_init, tuple_layers: bool = True):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from test1_b200.models.llama import LlamaConfig as OurCfg

    ours = getattr(OurCfg, model_name)()
    d = ours.to_hf_dict()
    for k in ("model_type", "architectures", "torch_dtype"):
        d.pop(k, None)
    hf_cfg = LlamaConfig(**d)
    attn = "flash_attention_2"
    try:
        import flash_attn  # noqa: F401
    except Exception:
        attn = "sdpa"
    hf_cfg._attn_implementation = attn
    try:
        from liger_kernel.transformers import apply_liger_kernel_to_llama

        apply_liger_kernel_to_llama()
    except Exception:
        pass
    with torch.device("meta"):
        model = LlamaForCausalLM(hf_cfg)
    model = model.to_empty(device="cpu").to(torch.bfloat16)
    # to_empty leaves non-persistent buffers (the rotary inv_freq) unset:
    # rebuild the rotary module from the config
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    model.model.rotary_emb = LlamaRotaryEmbedding(config=hf_cfg)
    gen = torch.Generator(device=device_for_init).manual_seed(42)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            else:
                r = torch.randn(p.shape, generator=gen, device=device_for_init, dtype=torch.float32)
                p.copy_((r * ours.initializer_range).to(torch.bfloat16).cpu())
    model.config._attn_implementation = attn
    return (_tuple_layers(model) if tuple_layers else model), attn


def run(args, rank, world, local):
    import torch
    import torch.distributed as dist

    if not os.path.isdir(REF) or not os.path.exists(os.path.join(REF, "slide_fsdp.py")):
        return {"unavailable": "reference source not present in baseline/_ref"}
    sys.path.insert(0, REF)
    try:
        from config import SlideFSDPConfig as RefConfig  # reference's own module
        from slide_fsdp import SlideFSDP as RefSlideFSDP
    except Exception as exc:  # pragma: no cover - depends on the box
        return {"unavailable": f"reference import failed: {type(exc).__name__}: {exc}"}

    dev = torch.device("cuda", local)
    t0 = time.time()
    model, attn = build_hf_model(args.model, "cpu")
    cfg = RefConfig(dtype=torch.bfloat16, device=dev, param_transfer_mode=args.param_transfer_mode,
                    grad_sync_mode=args.grad_sync_mode, gpu_buffer_pool_size=args.pool, lr=1e-5,
                    weight_decay=0.01, attention_implementation=attn, ac_offload_mode=args.ac_offload,
                    max_seq_length=args.seq, train_batch_size=args.batch)
    engine = RefSlideFSDP(model, cfg)
    init_s = time.time() - t0

    V = model.config.vocab_size
    g = torch.Generator().manual_seed(1000 + rank)
    n = args.warmup + 2 * args.steps
    batches = [torch.randint(0, V, (args.batch, args.seq), generator=g).pin_memory() for _ in range(n)]
    dev_batches = [b.to(dev) for b in batches]

    def drain():
        for st in engine.layer_states:
            st.wait_for_update()
        torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    losses = []
    for i in range(args.warmup):
        out = engine(input_ids=dev_batches[i], labels=dev_batches[i])
        losses.append(float(out.loss.detach()))
    drain()
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
        b = dev_batches[args.warmup + k]
        last = engine(input_ids=b, labels=b).loss
    drain()
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
            hb = batches[args.warmup + args.steps + k]
            ids = hb.to(dev, non_blocking=True)
            out = engine(input_ids=ids, labels=ids)
            losses.append(out.loss.item())
        drain()
        e_end.record()
        e_end.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
        tokens = args.batch * args.seq * world * args.steps
        e2e = {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": "tokens/s",
               "h2d_bytes_per_step": int(args.batch * args.seq * 8), "d2h_bytes_per_step": 4}
    return {"dev_ms": dev_ms, "e2e": e2e, "clocks": clocks, "launches": 0, "init_s": init_s,
            "losses": losses, "attn_implementation": attn}
