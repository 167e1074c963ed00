"""SlideFSDP: layer-sliding training with host-resident master weights.

Public API of the reference (slide_fsdp.py:116-745): ``SlideFSDP(model,
config)``; ``forward(input_ids, attention_mask=None, labels=None)`` runs the
forward pass *and* the backward pass and the per-layer optimizer updates,
and returns a ``CausalLMOutputWithPast``; ``update_learning_rate``,
``clip_grad_norm_``, ``save_pretrained``.  Added: ``save_state`` /
``load_state`` (fp32 master + optimizer state + step counters, which the
reference cannot save), ``close``.

Layer indexing is the reference's: 0 = embedding, 1..L = decoder layers,
L+1 = output layer (final norm + lm_head).

How a step runs (all GPU work is ordered by CUDA events; the host blocks only
on data dependencies):

  forward   for each layer: the copy stream loads layer i+1 into a free pool
            unit while layer i computes; the input of every decoder layer is
            checkpointed (kept, or offloaded to host memory on a side
            stream); the output layer computes loss and its own gradients in
            one pass (no logits kept for a later backward).
  backward  layers L..1 recompute from their checkpoint and run their
            explicit backward kernels; parameter gradients land in the pool
            unit; the gradient stream moves this rank's share to host memory
            (reduce-scatter / device-to-host copy, see parallel/comm.py); the
            host optimizer thread updates the shared fp32 master and writes
            the bf16 shadow that the next forward copies to the GPU.

Compared with the reference: no autograd hooks or per-layer autograd
Functions (so none of the hook-ordering races of slide_fsdp.py:416-430), no
per-pass fp32->bf16 CPU cast (the optimizer writes the shadow), the embedding
backward does not reload the embedding weights, and the optimizer is sharded
across ranks.
"""
from __future__ import annotations

import json
import math
import os
import time
import uuid
import warnings
import zlib
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _native, ops
from .config import SlideFSDPConfig
from .models import generic
from .models.llama import LlamaConfig, LlamaDecoderLayer, LlamaForCausalLM, make_context
from .optim.layer_adam import LayerAdam
from .parallel.comm import CpuReduceSlots, make_comm
from .runtime.activations import ActivationStore
from .runtime.device import Event, Stream
from .runtime import host_memory
from .runtime.host_memory import (REGION_HEADER_BYTES, HostRegion, MasterStore, RegionPlanner,
                                  check_region_header, write_region_header)
from .utils.trace import PhaseTracer
from .runtime.layer_state import (LayerBufferPool, LayerLayout, LayerRuntimeState, build_layout,
                                  shard_size)
from .runtime.update import UpdateScheduler

try:
    from transformers.modeling_outputs import CausalLMOutputWithPast
except Exception:  # pragma: no cover
    @dataclass
    class CausalLMOutputWithPast:  # type: ignore[no-redef]
        loss: Optional[torch.Tensor] = None
        logits: Optional[torch.Tensor] = None


class OutputLayer(nn.Module):
    """Final norm + lm_head moved as one unit (reference slide_fsdp.py:45-113).
    ``named_parameters``: norm.weight, lm_head.weight.

    With ``chunk_tokens`` > 0 (the default, from
    ``SlideFSDPConfig.lm_head_chunk_tokens``) the lm_head GEMM, the
    cross-entropy and both gradients run in chunks of that many tokens, so
    only a [chunk_tokens, V] logits buffer ever exists -- the role of
    Liger's fused linear cross-entropy in the reference
    (slide_fsdp.py:86-98); 0 materialises the full [T, V] logits."""

    def __init__(self, norm: nn.Module, lm_head: nn.Module, eps: float, chunk_tokens: int = 0):
        super().__init__()
        self.norm = norm
        self.lm_head = lm_head
        self.eps = eps
        self.chunk_tokens = int(chunk_tokens)

    def _grads(self):
        for p in self.parameters():
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        return self.norm.weight.grad, self.lm_head.weight.grad

    def loss_and_grad(self, h: torch.Tensor, ctx):
        """Forward + loss + backward of this layer.  Returns (loss, dh)."""
        w_n, w_lm = self.norm.weight.data, self.lm_head.weight.data
        x, rstd = ops.rmsnorm_fwd(h, w_n, self.eps)
        g_n, g_lm = self._grads()
        if self.chunk_tokens > 0:
            dx = torch.empty_like(x)
            loss, _ = ops.linear_cross_entropy(x, w_lm, ctx.targets, dx, g_lm, self.chunk_tokens)
        else:
            logits = ops.linear_fwd(x, w_lm)
            loss, dlogits, _ = ops.cross_entropy_fwd_bwd(logits, ctx.targets)
            del logits
            dx = ops.linear_dgrad(dlogits, w_lm)
            ops.linear_wgrad(dlogits, x, out=g_lm)
            del dlogits
        dh, dw = ops.rmsnorm_bwd(dx, h, w_n, rstd)
        g_n.copy_(dw)
        return loss, dh

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        x, _ = ops.rmsnorm_fwd(h, self.norm.weight.data, self.eps)
        return ops.linear_fwd(x, self.lm_head.weight.data)


def _convert_hf_llama(model: nn.Module) -> LlamaForCausalLM:
    """Build our Llama module from an HF LlamaForCausalLM, copying weights
    (names are identical)."""
    cfg = LlamaConfig.from_hf(model.config)
    ours = LlamaForCausalLM(cfg, device="meta")
    src = dict(model.named_parameters())
    for name, p in ours.named_parameters():
        if name not in src:
            raise ValueError(f"HF model lacks parameter {name}")
        if tuple(src[name].shape) != tuple(p.shape):
            raise ValueError(f"shape mismatch for {name}: {tuple(src[name].shape)} vs {tuple(p.shape)}")
        p.data = src[name].data
    return ours


class SlideFSDP(nn.Module):
    def __init__(self, model: nn.Module, config: SlideFSDPConfig):
        super().__init__()
        self.config = config
        self.device = torch.device(config.device)
        self.init_times: Dict[str, float] = {}  # seconds per set-up phase
        t_phase = [time.perf_counter()]

        def phase(name: str) -> None:
            now = time.perf_counter()
            self.init_times[name] = round(now - t_phase[0], 3)
            t_phase[0] = now

        self.dtype = config.dtype
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.world_size = dist.get_world_size() if dist.is_initialized() else 1
        self.is_cuda = self.device.type == "cuda"
        local_ranks = int(os.environ.get("LOCAL_WORLD_SIZE", str(self.world_size)) or self.world_size)
        if self.world_size > 1 and local_ranks < self.world_size:
            # the master weights and the update counters live in one node's
            # shared host memory (as the reference's /dev/shm files do)
            raise NotImplementedError(
                f"SlideFSDP runs on one node: WORLD_SIZE={self.world_size} but LOCAL_WORLD_SIZE={local_ranks}")
        if self.is_cuda:
            torch.cuda.set_device(self.device)
        elif "OMP_NUM_THREADS" not in os.environ:
            # CPU ranks compute with torch's intra-op pool; N ranks on one
            # host with a full-size pool each oversubscribe the cores (spinning
            # OpenMP workers slow every op by ~40x).  torchrun sets
            # OMP_NUM_THREADS=1; other launchers get the rank's share here.
            local_world = int(os.environ.get("LOCAL_WORLD_SIZE", "1") or 1)
            if local_world > 1:
                torch.set_num_threads(max(1, len(os.sched_getaffinity(0)) // local_world))
        _native.host()  # load + size the host worker pool
        if config.host_threads > 0:
            _native.host().configure_threads(config.host_threads, _native._cpu_list_from_env())

        # Llama-structured models run the sm_100a layer programs; any other
        # HF causal LM runs its own modules under autograd (models/generic.py)
        self.generic = False
        if not isinstance(model, LlamaForCausalLM):
            if generic.is_native_llama(model):
                model = _convert_hf_llama(model)
            else:
                self.generic = True
        if getattr(model.config, "tie_word_embeddings", False):
            raise NotImplementedError("tied input/output embeddings are not supported by layer sliding")
        if not self.generic and config.use_native_kernels and self.dtype != torch.bfloat16:
            # fail here rather than at the first kernel of the first step
            raise NotImplementedError(
                f"the sm_100a Llama kernels compute in bfloat16; dtype={self.dtype} runs on the "
                f"generic layer path (other HF architectures) or with use_native_kernels=False")
        self.base_model = model
        self.model_config = model.config
        self._split_model(model)
        phase("split_model")

        # ---- communication -------------------------------------------------
        self.comm = None  # built after the shared region exists (cpu_reduce slots live there)
        self._session = self._make_session_id()

        # ---- layouts -------------------------------------------------------
        self.layouts: List[LayerLayout] = []
        for idx, (kind, mod) in enumerate(self._layer_modules()):
            self.layouts.append(build_layout(idx, kind, getattr(mod, "params_root", mod)))
        if self.generic:
            for l in self.layouts:
                for e in l.entries:
                    e.hf_name = self._hf_names[id(e.param)]
        self.num_layers = len(self.layouts)
        self.total_params = sum(l.numel for l in self.layouts)
        self.max_param_size = max(l.numel for l in self.layouts)

        # ---- shared host region: counters | master fp32 | shadow bf16 | cpu slots
        plan = RegionPlanner(align=4096)
        self._hdr_off = plan.take(REGION_HEADER_BYTES)
        n_counters = 4 * self.num_layers + 64
        self._ctr_off = plan.take(8 * n_counters)
        self.split_master = self.dtype == torch.bfloat16 and config.master_layout == "split"
        if self.dtype == torch.bfloat16 and config.master_layout == "bf16":
            self.master_layout = "bf16"
        else:
            self.master_layout = "split" if self.split_master else "fp32"
        want_shadow = self.dtype != torch.float32
        for l in self.layouts:
            mb, _ = MasterStore.bytes_needed(l.numel, self.split_master, want_shadow, self.master_layout)
            l.master_off = plan.take(mb)
        for l in self.layouts:
            _, sb = MasterStore.bytes_needed(l.numel, self.split_master, want_shadow, self.master_layout)
            l.shadow_off = plan.take(sb) if sb else None
        dec_caps = [l.numel for l in self.layouts if l.kind == "decoder"]
        big_caps = [l.numel for l in self.layouts if l.kind != "decoder"]
        # slot capacity rounded to 4096 elements: every slot starts on a page
        self._slot_cap = -(-max(dec_caps + big_caps) // 4096) * 4096
        self._n_slots = 4
        self._slots_off = None
        if self.world_size > 1 and config.grad_sync_mode == "cpu_reduce":
            es = torch.tensor([], dtype=self.dtype).element_size()
            self._slots_off = plan.take(CpuReduceSlots.region_bytes(self._slot_cap, self.world_size,
                                                                    self._n_slots, es))
        shm_path = None
        if self.world_size > 1:
            shm_path = f"/dev/shm/t1b200_{self._session}.bin"
        self._check_host_capacity(plan.size, shm_path)
        creator = self.rank == 0
        if self.world_size > 1 and not creator:
            dist.barrier()
        self.shared = HostRegion(plan.size, shm_path=shm_path, create=creator or shm_path is None,
                                 pin=False)
        header = self._region_fields(plan.size)
        if creator:
            write_region_header(self.shared, self._hdr_off, header)
        if self.world_size > 1 and creator:
            dist.barrier()
        if not creator:
            check_region_header(self.shared, self._hdr_off, header, self.rank)
        if self.world_size > 1:
            dist.barrier()  # every local rank has mapped the region
            if creator:
                self.shared.unlink()
        self.counters = self.shared.view(torch.uint8, self._ctr_off, 8 * n_counters)
        # step-entry heartbeat: counter[base + r] = steps rank r has started,
        # counter[base + 32 + r] = 1 + the steps rank r completed before it
        # left (0 while it is still training)
        self._live_base = 4 * self.num_layers
        phase("shared_region")

        # ---- comm strategy (needs the slot region for cpu_reduce)
        cpu_slots = None
        if self._slots_off is not None:
            slot_region = _SubRegion(self.shared, self._slots_off)
            cpu_slots = CpuReduceSlots(slot_region, self.counters, 2 * self.num_layers, self.num_layers,
                                       self._slot_cap, self.rank, self.world_size, self._n_slots,
                                       timeout_s=config.host_wait_timeout_s, dtype=self.dtype)
        self.cpu_slots = cpu_slots
        self.comm = make_comm(config, self.device, self.rank, self.world_size, cpu_slots)
        phase("comm")

        # ---- master stores; init (rank 0 writes), then everyone pins
        self.stores = [MasterStore(self.shared, l.numel, l.master_off, self.split_master, self.dtype,
                                   l.shadow_off, layout=self.master_layout) for l in self.layouts]
        self._place_master_shards()
        self._init_master(model)
        if self.world_size > 1:
            dist.barrier()
        phase("master_init")

        # ---- per-rank host gradients (this rank's update range of each layer)
        gplan = RegionPlanner(align=4096)
        self._grad_offs = []
        for l in self.layouts:
            s, e = self.comm.update_range(l.numel)
            gbytes = torch.tensor([], dtype=self.dtype).element_size()
            self._grad_offs.append((gplan.take(gbytes * max(e - s, 0)), max(e - s, 0)))
        self.grad_region = HostRegion(max(gplan.size, 4096), pin=False)
        grad_unpinned = []
        if self.is_cuda:
            gb = torch.tensor([], dtype=self.dtype).element_size()
            grad_unpinned = self.grad_region.pin([(off, n * gb) for off, n in self._grad_offs if n],
                                                 strict=False)
        phase("grad_region")

        # ---- runtime states
        self.layer_states: List[LayerRuntimeState] = []
        for l, (kind, mod), store in zip(self.layouts, self._layer_modules(), self.stores):
            goff, gn = self._grad_offs[l.idx]
            grad_host = self.grad_region.view(self.dtype if self.dtype != torch.float32 else torch.float32,
                                              goff, gn) if gn else None
            st = LayerRuntimeState(l, mod, store.bind_tensor, store.shadow, grad_host,
                                   self.comm.update_range(l.numel))
            st.store = store
            st.bind_host()
            self.layer_states.append(st)

        # ---- page-lock what this rank's GPU reads or writes in the shared region
        shared_unpinned = []
        if self.is_cuda:
            shared_unpinned = self.shared.pin(self._pin_ranges(), strict=False)
        self._pin_fallback(shared_unpinned, grad_unpinned)
        phase("pin_shared")

        # ---- optimizer (this rank's range of every layer)
        self.layer_optimizer = self._create_optimizer(config)
        phase("optimizer")

        # ---- GPU buffer pools
        alloc = self.comm.allocator(self.dtype)
        self.pool = LayerBufferPool(max(self.comm.unit_capacity(c) for c in dec_caps) if dec_caps else 1,
                                    self.dtype, self.device, config.gpu_buffer_pool_size,
                                    allocator=alloc, name="decoder-pool")
        self.big_pool = LayerBufferPool(max(self.comm.unit_capacity(c) for c in big_caps),
                                        self.dtype, self.device, 1, allocator=alloc,
                                        name="embed/output-unit")
        for st in self.layer_states:
            st.pool = self.pool if st.kind == "decoder" else self.big_pool
        phase("gpu_pools")

        # ---- streams, scheduler, activations
        self.h2d_stream = Stream(self.device)
        self.grad_stream = Stream(self.device)
        self.ac_d2h = Stream(self.device)
        self.updates = UpdateScheduler(self.counters, timeout_s=config.host_wait_timeout_s)
        self._reducer = (UpdateScheduler(self.counters, name="t1-reduce", fifo=True,
                                         timeout_s=config.host_wait_timeout_s)
                         if cpu_slots is not None else None)
        self.acts = ActivationStore(config.ac_offload_mode if config.enable_activation_checkpoint else "gpu",
                                    self.device, self.ac_d2h, self.h2d_stream, config.ac_offload_dir)
        trace = config.trace_path or os.environ.get("T1_TRACE") or None
        if trace and self.world_size > 1:
            trace = f"{trace}.rank{self.rank}"
        self.tracer = PhaseTracer(self.device, trace, self.rank, self.world_size)
        self.completed_steps = 0
        self.stats: Dict[str, float] = {}
        # exact gradient clipping: per-layer squared norms and the deferred
        # updates of the current step
        self._exact_clip = bool(config.exact_grad_clip and config.clip_grad_norm > 0)
        self._clip_parts: Dict[int, float] = {}
        self._deferred: Dict[int, tuple] = {}
        self.last_grad_norm: Optional[float] = None
        self.h2d_bytes = 0
        self.position_embeddings = None
        self._closed = False
        if self.rank == 0 and os.environ.get("T1_QUIET", "0") != "1":
            self._print_model_info()

    # ------------------------------------------------------------ set-up
    def _pin_ranges(self) -> list:
        """(offset, bytes) ranges of the shared region that this rank's GPU
        touches: the host tensors its parameter fetches read (every layer's
        bf16 copy in ``full`` mode, only its own shard in ``shard`` mode) and
        the cpu_reduce slots.  Rounded out to pages and merged, so no two
        registrations share a page and each copy lies in one registration.
        Every local rank maps the same pages, so pinning only what each
        rank reads keeps the node's page-locked total near one copy of the
        model instead of one per GPU."""
        base = self.shared.buf.data_ptr()
        spans = []
        for st in self.layer_states:
            for t in self.comm.host_read_views(st):
                if t.numel():
                    off = t.data_ptr() - base
                    spans.append((off, off + t.numel() * t.element_size()))
        if self._slots_off is not None:
            es = torch.tensor([], dtype=self.dtype).element_size()
            n = CpuReduceSlots.region_bytes(self._slot_cap, self.world_size, self._n_slots, es)
            spans.append((self._slots_off, self._slots_off + n))
        page = 4096
        spans = sorted((a // page * page, min(-(-b // page) * page, self.shared.nbytes)) for a, b in spans)
        merged = []
        for a, b in spans:
            if merged and a <= merged[-1][1]:
                merged[-1][1] = max(merged[-1][1], b)
            else:
                merged.append([a, b])
        return [(a, b - a) for a, b in merged]

    def _check_host_capacity(self, shared_bytes: int, shm_path: Optional[str]) -> None:
        """Refuse, on every rank alike and before anything is allocated, a
        configuration whose host memory does not fit this node: an
        over-committed node kills ranks (or its other jobs) in the middle of
        a run, and a shared-memory file larger than its mount faults on
        first touch.  Counts the shared master, every local rank's gradient
        shards and optimizer state."""
        c = self.config
        local = int(os.environ.get("LOCAL_WORLD_SIZE", str(self.world_size)) or 1)
        es = torch.tensor([], dtype=self.dtype).element_size()
        sb = 2 if c.optimizer_state_dtype == "bf16" else 4
        if self.world_size > 1 and c.optimizer_sharding == "rank0":
            owned = self.total_params  # one optimizer and gradient copy on the node
        else:
            owned = self.total_params * min(local, self.world_size) / self.world_size
        need = shared_bytes + owned * (2 * sb + es)
        avail = host_memory.mem_available_bytes()
        problems = []
        if avail is not None and need > avail:
            problems.append(f"host memory: {need / 1e9:.1f} GB needed (master {shared_bytes / 1e9:.1f} GB, "
                            f"optimizer state and gradients {owned * (2 * sb + es) / 1e9:.1f} GB for "
                            f"{min(local, self.world_size)} local rank(s)), {avail / 1e9:.1f} GB available")
        if shm_path is not None:
            free = host_memory.shm_free_bytes(os.path.dirname(shm_path))
            if free is not None and shared_bytes > free:
                problems.append(f"{os.path.dirname(shm_path)}: {shared_bytes / 1e9:.1f} GB needed, "
                                f"{free / 1e9:.1f} GB free")
        bad = torch.tensor([1.0 if problems else 0.0], device=self.device)
        if self.world_size > 1:
            dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if bad.item() > 0:
            detail = "; ".join(problems) if problems else "another rank found too little host memory"
            raise MemoryError(f"rank {self.rank}: this model and configuration do not fit on the node: {detail} "
                              f"(bf16 optimizer state, master_layout='bf16' or more nodes reduce it)")

    def _region_fields(self, nbytes: int) -> dict:
        """What the shared region's layout depends on, for its header."""
        c = self.config
        desc = (f"{self.master_layout}|{self.dtype}|{c.param_transfer_mode}|{c.grad_sync_mode}|"
                f"{c.optimizer_sharding}|{[l.numel for l in self.layouts]}")
        return {"region_bytes": nbytes, "world_size": self.world_size, "num_layers": self.num_layers,
                "total_params": self.total_params, "layout_code": zlib.crc32(desc.encode())}

    def _numa_node(self) -> Optional[int]:
        """NUMA node of this rank's GPU: ``NUMA_NODE`` from the launcher, else
        sysfs through the device's PCI address."""
        from .runtime import numa

        if os.environ.get("NUMA_NODE", "").isdigit():
            return int(os.environ["NUMA_NODE"])
        if not self.is_cuda:
            return None
        p = torch.cuda.get_device_properties(self.device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        return numa.gpu_numa_node(0, bus_ids=[bus])

    def _place_master_shards(self) -> None:
        """On hosts with several NUMA nodes, before rank 0 first touches the
        shared master, every rank gives the pages of its own optimizer shard
        (the planes its LayerAdam threads stream every step) a preferred
        placement on its GPU's node.  The policy lives on the shared-memory
        object, so it applies whichever process faults the pages in.  A
        no-op on single-node hosts."""
        from .runtime import numa

        nodes = numa.numa_nodes()
        if len(nodes) > 1:
            node = self._numa_node()
            if node is not None and node in nodes:
                host = _native.host()
                for l, store in zip(self.layouts, self.stores):
                    s, e = self.comm.update_range(l.numel)
                    if e <= s:
                        continue
                    sl = store.optim_slice(s, e)
                    for t in (sl if isinstance(sl, tuple) else (sl,)):
                        host.numa_bind(t, [node], "preferred")
        if self.world_size > 1:
            dist.barrier()  # every policy is set before the first touch

    def _pin_fallback(self, shared_unpinned: list, grad_unpinned: list) -> None:
        """Host ranges the OS refused to page-lock stay pageable: plain
        copies from them still work (driver-staged, slower), but the fused
        kernels map host memory directly, so if any rank lost a range they
        need, every rank switches that path to the NCCL baseline."""
        if not self.is_cuda:
            return
        if shared_unpinned or grad_unpinned:
            print(f"[rank {self.rank}] warning: {len(shared_unpinned)} shared and {len(grad_unpinned)} "
                  f"gradient host ranges could not be page-locked; copies from them are staged",
                  flush=True)
        flags = torch.tensor([1.0 if shared_unpinned else 0.0, 1.0 if grad_unpinned else 0.0],
                             device=self.device)
        if self.world_size > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MAX)
        lost_params, lost_grads = (bool(x) for x in flags.tolist())
        if (lost_params or lost_grads) and hasattr(self.comm, "disable_fused"):
            self.comm.disable_fused(params=lost_params, grads=lost_grads)
            if self.rank == 0:
                print(f"fused NVLink paths disabled for: {'params ' if lost_params else ''}"
                      f"{'grads' if lost_grads else ''} (host memory not page-locked)", flush=True)

    def _make_session_id(self) -> str:
        sid = [uuid.uuid4().hex[:12]]
        if self.world_size > 1:
            dist.broadcast_object_list(sid, src=0)
        return sid[0]

    def _split_model(self, model: nn.Module) -> None:
        """embedding | decoder layers | (final norm + lm_head), as the
        reference splits any HF model (slide_fsdp.py:213-244)."""
        decoder = model.get_decoder()
        if hasattr(decoder, "layers"):
            layers = decoder.layers
        elif hasattr(decoder, "block"):
            layers = decoder.block
        else:
            raise ValueError("Cannot find decoder layers in model")
        self.num_decoder_layers = len(layers)
        self.rotary_emb = None
        if not self.generic:
            self.embed_tokens = model.get_input_embeddings()
            self.decoder_layers = nn.ModuleList(layers)
            self.output_layer = OutputLayer(decoder.norm, model.get_output_embeddings(),
                                            model.config.rms_norm_eps, self.config.lm_head_chunk_tokens)
            return
        self.embed_tokens = generic.GenericEmbedding(model.get_input_embeddings())
        self.decoder_layers = nn.ModuleList(generic.GenericDecoderLayer(l) for l in layers)
        self.output_layer = generic.GenericOutputLayer(decoder.norm, model.get_output_embeddings())
        rot = getattr(decoder, "rotary_emb", None)
        if rot is not None:
            # a fresh instance on the compute device (its buffers are not
            # parameters, and a deferred-init model has them on meta)
            self.rotary_emb = type(rot)(model.config, device=self.device)
        # HF names of every parameter, for checkpoints of any architecture
        self._hf_names = {id(p): n for n, p in model.named_parameters()}

    def _make_context(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor]):
        if not self.generic:
            return make_context(self.model_config, input_ids, labels, self.device)
        B, S = input_ids.shape
        ids = input_ids.to(self.device, non_blocking=True)
        pos = torch.arange(S, device=self.device).unsqueeze(0)
        pe = None
        if self.rotary_emb is not None:
            x = torch.empty(1, S, 1, device=self.device, dtype=self.dtype)
            pe = self.rotary_emb(x, pos)
        tg = ops.shift_labels(labels.to(self.device, non_blocking=True)) if labels is not None else None
        masks = generic.causal_masks(self.model_config, B, S, self.model_config.hidden_size, pos,
                                     self.device, self.dtype)
        return generic.GenericContext(B, S, pe, pos, ids, tg, masks)

    def _layer_modules(self):
        out = [("embed", self.embed_tokens)]
        out += [("decoder", l) for l in self.decoder_layers]
        out.append(("output", self.output_layer))
        return out

    @property
    def all_layers(self):
        return [m for _, m in self._layer_modules()]

    def _create_optimizer(self, config: SlideFSDPConfig) -> Optional[LayerAdam]:
        opt = LayerAdam(lr=config.lr, betas=config.adam_betas, eps=config.adam_eps,
                        weight_decay=config.weight_decay, bias_correction=config.bias_correction,
                        adamw_mode=True, fp32_optimizer_state=True, num_layer=self.num_layers,
                        nvme_offload_fraction=config.optimizer_nvme_offload_fraction,
                        offload_dir=config.optimizer_offload_dir, prefetch=True,
                        state_dtype=torch.bfloat16 if config.optimizer_state_dtype == "bf16" else None)
        n = 0
        for st in self.layer_states:
            s, e = st.shard
            if e > s:
                opt.add_flat_layer(st.idx, st.store.optim_slice(s, e))
                n += 1
        return opt if n else None

    @torch.no_grad()
    def _init_master(self, model: nn.Module) -> None:
        """Rank 0 fills the shared fp32 master from the model's parameters
        (random N(0, initializer_range) when they are on the meta device),
        then writes the low-precision shadow."""
        if self.rank != 0:
            return
        host = _native.host()
        std = self.model_config.initializer_range
        seed = self.config.seed
        gen_dev = self.device if self.is_cuda else torch.device("cpu")
        chunk = 1 << 26
        staging = torch.empty(chunk, dtype=torch.float32, pin_memory=self.is_cuda)
        for l, store in zip(self.layouts, self.stores):
            for k, e in enumerate(l.entries):
                p = e.param
                if p.device.type == "meta":
                    const = None
                    if e.name.endswith("norm.weight") or e.name.endswith("layernorm.weight"):
                        const = 1.0
                    elif e.name.endswith(".bias"):
                        const = 0.0
                    if const is not None:
                        for c0 in range(0, e.numel, chunk):
                            c1 = min(e.numel, c0 + chunk)
                            store.write_fp32(staging[: c1 - c0].fill_(const), e.offset + c0)
                    else:
                        g = torch.Generator(device=gen_dev)
                        g.manual_seed(seed * 1_000_003 + l.idx * 7919 + k)
                        for c0 in range(0, e.numel, chunk):
                            c1 = min(e.numel, c0 + chunk)
                            r = torch.randn(c1 - c0, generator=g, device=gen_dev, dtype=torch.float32)
                            staging[: c1 - c0].copy_(r.mul_(std))
                            store.write_fp32(staging[: c1 - c0], e.offset + c0)
                else:
                    store.write_fp32(p.detach().reshape(-1).float(), e.offset)

    def _print_model_info(self) -> None:
        gb = 1e9
        print("=" * 60)
        print("SlideFSDP (test1_b200) model info")
        print("=" * 60)
        print(f"Model type: {self.model_config.model_type}")
        print(f"Num decoder layers: {self.num_decoder_layers}")
        print(f"Total parameters: {self.total_params:,}")
        print(f"Max layer param size: {self.max_param_size:,}")
        print(f"Param transfer mode: {self.config.param_transfer_mode}")
        print(f"Grad sync mode: {self.config.grad_sync_mode}  (optimizer sharding: {self.config.optimizer_sharding})")
        print(f"World size: {self.world_size}   comm: {self.comm.name}")
        print(f"Host memory: master {self.total_params * 4 / gb:.2f} GB, shadow {self.total_params * 2 / gb:.2f} GB, "
              f"optimizer state (this rank) {self._opt_numel() * 8 / gb:.2f} GB")
        print(f"GPU buffer pool: {self.config.gpu_buffer_pool_size} units x {self.pool.capacity:,} elements "
              f"+ 1 embed/output unit x {self.big_pool.capacity:,}")
        print(f"Host SIMD: {_native.host().simd_level()}  threads: {_native.host().num_threads()}")
        print("Set-up (s): " + ", ".join(f"{k} {v:.1f}" for k, v in self.init_times.items()))
        print("=" * 60, flush=True)

    def _opt_numel(self) -> int:
        return sum(max(0, st.shard[1] - st.shard[0]) for st in self.layer_states)

    # ------------------------------------------------------ layer movement
    def _update_target(self, st: LayerRuntimeState) -> int:
        return self.comm.updaters_for(st.numel) * self.completed_steps

    def _fetch(self, st: LayerRuntimeState, with_grad: bool, need_weights: bool = True,
               host_leg_only: bool = False) -> None:
        """Acquire a pool unit for ``st`` and enqueue its parameter load.
        ``host_leg_only``: staged shard mode with the gather fused into the
        QKV GEMM -- enqueue only the copy-engine transfer of this rank's
        shard; the layer's fused kernel broadcasts it."""
        if st.resident:
            if with_grad:
                st.bind_device(with_grad=True)
            return
        unit = st.pool.acquire(st.idx)
        st.unit = unit
        if need_weights:
            # the previous step's optimizer update of this layer must be visible
            t0 = time.perf_counter()
            self.updates.wait_counter(st.idx, self._update_target(st))
            self.tracer.host("wait_update", st.idx, time.perf_counter() - t0)
            self.h2d_stream.wait(unit.free_event)
            tok = self.tracer.begin("h2d", st.idx, self.h2d_stream)
            if host_leg_only:
                self.comm.fetch_host_leg(st, unit.param, self.h2d_stream)
                st.gather_pending = True
            else:
                self.comm.fetch_params(st, unit.param, self.h2d_stream)
            self.tracer.end(tok)
            self.h2d_bytes += self.comm.h2d_bytes(st, unit.param.element_size())
            st.loaded = self.h2d_stream.record()
        else:
            st.loaded = unit.free_event
        st.bind_device(with_grad=with_grad)

    def _acquire_unloaded(self, st: LayerRuntimeState) -> None:
        """Take a pool unit for ``st`` whose weights a fused kernel on the
        compute stream will load; the compute stream waits until the unit's
        previous occupant is done with it."""
        self.updates.wait_counter(st.idx, self._update_target(st))
        unit = st.pool.acquire(st.idx)
        st.unit = unit
        if unit.free_event is not None and unit.free_event.e is not None:
            torch.cuda.current_stream(self.device).wait_event(unit.free_event.e)
        st.loaded = None
        st.bind_device(with_grad=False)
        self.h2d_bytes += self.comm.h2d_bytes(st, unit.param.element_size())

    def _check_unit(self, st: LayerRuntimeState, where: str) -> None:
        """Debug aid (env T1_CHECK_FETCH=1): compare the device copy of a
        layer with the bf16 rounding of its host master and report elements
        that differ by more than one bf16 ulp."""
        if os.environ.get("T1_CHECK_FETCH", "0") != "1" or st.unit is None or not self.is_cuda:
            return
        torch.cuda.synchronize(self.device)
        dev = st.unit.param[: st.numel].float().cpu()
        ref = st.store.read_fp32().bfloat16().float()
        tol = ref.abs() * 2.0 ** -7 + 1e-30
        bad = (dev - ref).abs() > tol
        n = int(bad.sum())
        if n:
            idx = bad.nonzero()[:4].flatten().tolist()
            print(f"[rank {self.rank}] T1_CHECK_FETCH {where} layer {st.idx}: {n} of {st.numel} elements differ "
                  f"(first at {idx}: dev {[dev[i].item() for i in idx]} ref {[ref[i].item() for i in idx]})",
                  flush=True)

    def _early_weight(self, st: LayerRuntimeState, name: str) -> torch.Tensor:
        """One small parameter of layer ``st`` on the device ahead of the
        layer's fused gather, with exactly the values the gather delivers (so
        the forward and the backward recompute agree): the bf16 copy when the
        fetch is staged, else the fp32 master rounded to nearest even as the
        gather kernel rounds it."""
        for e in st.layout.entries:
            if e.name == name:
                if getattr(self.comm, "staged", False):
                    w = st.shadow[e.offset:e.offset + e.numel].view(e.shape)
                else:
                    w = st.store.read_fp32(e.offset, e.offset + e.numel).to(self.dtype).view(e.shape)
                if not self.is_cuda:
                    return w
                # through page-locked staging (torch's caching host allocator
                # keeps it alive until the copy ran), so the host never waits
                return w.pin_memory().to(self.device, non_blocking=True)
        raise KeyError(f"layer {st.idx} has no parameter {name}")

    def _wait_loaded(self, st: LayerRuntimeState) -> None:
        if st.loaded is not None and st.loaded.e is not None:
            torch.cuda.current_stream(self.device).wait_event(st.loaded.e)
        st.loaded = None

    def _release(self, st: LayerRuntimeState, done: Event) -> None:
        st.pool.release(st.unit, done)
        st.unit = None
        st.bind_host()

    def _grad_ready_hook(self, st: LayerRuntimeState):
        """Per-tensor gradient sync during a decoder layer's backward (fused
        NVLink reduce-scatter only): each weight gradient starts its
        reduce-scatter + host store on the gradient stream as soon as it is
        final, overlapping the rest of the layer's backward."""
        if not getattr(self.comm, "grads_by_range", False) or st.unit is None:
            return None
        base = st.unit.grad.data_ptr()
        es = st.unit.grad.element_size()
        st.synced = []

        def ready(t: torch.Tensor) -> None:
            lo = (t.data_ptr() - base) // es
            hi = lo + t.numel()
            self.grad_stream.wait(Event(self.device).record())
            tok = self.tracer.begin("grad_sync", st.idx, self.grad_stream)
            self.comm.sync_grads_range(st, st.unit.grad, self.grad_stream, lo, hi)
            self.tracer.end(tok)
            st.synced.append((lo, hi))

        return ready

    def _offload_grads(self, st: LayerRuntimeState, step: int) -> None:
        """After the backward of ``st``: move gradients to the host, free
        the unit, schedule the optimizer update."""
        computed = Event(self.device).record()
        self.grad_stream.wait(computed)
        unit = st.unit
        tok = self.tracer.begin("grad_sync", st.idx, self.grad_stream)
        synced = getattr(st, "synced", None)
        if synced:
            # the ranges not synced during the backward (the norm weights)
            pos = 0
            for lo, hi in sorted(synced):
                if lo > pos:
                    self.comm.sync_grads_range(st, unit.grad, self.grad_stream, pos, lo)
                pos = max(pos, hi)
            if pos < st.numel:
                self.comm.sync_grads_range(st, unit.grad, self.grad_stream, pos, st.numel)
            st.synced = []
        else:
            self.comm.sync_grads(st, unit.grad, self.grad_stream)
        self.tracer.end(tok)
        ready = self.grad_stream.record()
        self._release(st, ready)
        self._schedule_update(st, ready, step)

    def _schedule_update(self, st: LayerRuntimeState, ready: Event, step: int) -> None:
        opt = self.layer_optimizer
        s, e = st.shard
        has_work = opt is not None and e > s
        scale = self.comm.grad_scale
        lr = self.config.lr  # the rate of the step that produced these gradients
        shadow = (st.shadow[s:e] if (has_work and st.store.layout == "fp32" and self.dtype != torch.float32)
                  else None)

        def run_update(grad=None, coef=1.0):
            if has_work:
                g = grad if grad is not None else st.grad_host
                t0 = time.perf_counter()
                opt.step_flat(st.idx, g, shadow=shadow, grad_scale=scale * coef, lr=lr)
                self.tracer.host("adam", st.idx, time.perf_counter() - t0)
            if e > s:  # only ranks that own a slice publish
                self.updates.publish(st.idx)

        if self._exact_clip:
            # measure now, update once the global norm is known
            def measure(grad=None):
                g = grad if grad is not None else st.grad_host
                sq = 0.0
                if has_work and g is not None and g.numel():
                    sq = _native.host().sumsq(g) * scale * scale
                self._clip_parts[st.idx] = sq
                self._deferred[st.idx] = (run_update, grad)

            if self._reducer is not None:
                self._reducer.submit(st.idx, ready, lambda: measure(self.comm.host_reduce(st, step)))
            else:
                self.updates.submit(st.idx, ready, measure)
            return

        if self._reducer is not None:
            def run_reduce():
                g = self.comm.host_reduce(st, step)
                self.updates.submit(st.idx, None, lambda: run_update(g))
            self._reducer.submit(st.idx, ready, run_reduce)
        else:
            self.updates.submit(st.idx, ready, run_update)

    # -------------------------------------------------------------- step
    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                labels: Optional[torch.Tensor] = None, **kwargs) -> CausalLMOutputWithPast:
        if attention_mask is not None:
            self._check_mask(attention_mask)
        self._check_ids(input_ids, labels)
        if labels is None:
            return CausalLMOutputWithPast(loss=None, logits=self._inference(input_ids))
        loss = self._train_step(input_ids, labels)
        return CausalLMOutputWithPast(loss=loss, logits=None)

    def _check_ids(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor]) -> None:
        """Token ids and labels that arrive in host memory are range-checked
        before they are copied (device-resident ones are not, as that would
        synchronise every step; the kernels never access memory for an
        out-of-range id, and the bounds-checked build records it)."""
        V = self.model_config.vocab_size
        if input_ids.device.type == "cpu" and input_ids.numel():
            lo, hi = int(input_ids.min()), int(input_ids.max())
            if lo < 0 or hi >= V:
                raise ValueError(f"input_ids must lie in [0, {V}), got [{lo}, {hi}]")
        if labels is not None and labels.device.type == "cpu" and labels.numel():
            valid = labels[labels != -100]
            if valid.numel() and (int(valid.min()) < 0 or int(valid.max()) >= V):
                raise ValueError(f"labels must be -100 or lie in [0, {V})")

    def _check_mask(self, mask: torch.Tensor) -> None:
        """Causal attention without a mask is exact for right padding (no
        real token attends to a later pad token; pad positions carry label
        -100).  Other masks are rejected."""
        m = mask.bool()
        if bool(m.all()):
            return
        # right padding: once a row turns False it stays False
        if bool((m[:, 1:] & ~m[:, :-1]).any()):
            raise NotImplementedError("only right-padded attention masks are supported")

    def _enter_step(self, step: int) -> None:
        """Announce that this rank starts ``step`` and wait (bounded by
        ``host_wait_timeout_s``) until every other rank has started it too,
        before any GPU work or collective of the step is issued.  A rank that
        closed its engine is reported at once; one that stopped without
        closing is reported when the wait expires.  Either way the error
        names the rank, and nothing of this step is in flight on the GPU."""
        if self.world_size == 1 or self.world_size > 32:
            return
        host = _native.host()
        base = self._live_base
        host.counter_add(self.counters, base + self.rank, 1)
        timeout = float(self.config.host_wait_timeout_s)
        deadline = time.monotonic() + timeout
        for r in range(self.world_size):
            if r == self.rank:
                continue
            while host.counter_load(self.counters, base + r) < step:
                left = int(host.counter_load(self.counters, base + 32 + r))
                if left:
                    raise RankLeftError(f"rank {r} left the run after step {left - 1}; rank {self.rank} "
                                        f"cannot start step {step}")
                if time.monotonic() > deadline:
                    raise TimeoutError(f"rank {r} did not start step {step} within {timeout:.1f}s "
                                       f"(it stalled or died); rank {self.rank} stops before the step")
                host.counter_wait_geq(self.counters, base + r, step, 0.05)

    @torch.no_grad()
    def _train_step(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        cfg = self.model_config
        dev = self.device
        step = self.completed_steps + 1
        self._enter_step(step)
        if self.cpu_slots is not None:
            self.cpu_slots.step = step
        ctx = self._make_context(input_ids, labels)
        S = self.layer_states
        L = self.num_decoder_layers
        emb, out = S[0], S[L + 1]

        # ---------------- forward
        self._fetch(emb, with_grad=False)
        fuse_first = (L > 0 and not self.generic and hasattr(self.comm, "can_fuse_qkv")
                      and self.comm.can_fuse_qkv(S[1]) and self.config.use_native_kernels
                      and self.config.fuse_gather_qkv)
        # staged + fused: the copy engine brings this rank's shard of layer
        # i+1 into its unit while layer i computes; layer i+1's QKV kernel
        # then only pushes it to the peers
        staged = fuse_first and getattr(self.comm, "staged", False)
        prefetching = not fuse_first or staged
        if L > 0 and prefetching:
            self._fetch(S[1], with_grad=False, host_leg_only=staged)
        self._wait_loaded(emb)
        self._check_unit(emb, "forward")
        with self.tracer.span("fwd", 0):
            h = emb.module.forward_ids(ctx.input_ids)
        self._release(emb, Event(dev).record())
        prefetch = max(1, min(self.config.prefetch_layers, self.config.gpu_buffer_pool_size - 1))
        fuse_qkv = fuse_first
        cfgm = self.model_config
        n_qkv = cfgm.q_size + 2 * cfgm.kv_size if fuse_qkv else 0
        saved_all = {}
        for i in range(1, L + 1):
            st = S[i]
            qkv_fn = None
            ln1 = None
            if fuse_qkv and (getattr(st, "gather_pending", False) or not st.resident):
                # shard mode: the layer is gathered by its own fused QKV kernel;
                # the input norm ahead of it gets its weight separately
                if staged:
                    self._wait_loaded(st)  # this rank's shard is in the unit
                else:
                    self._acquire_unloaded(st)
                st.gather_pending = False
                qkv_fn = (lambda x1, rope, st=st: self.comm.ag_qkv(st, x1, n_qkv, rope))
                ln1 = self._early_weight(st, "input_layernorm.weight")
            else:
                self._wait_loaded(st)
            tok = self.tracer.begin("fwd", i)
            if self.config.enable_activation_checkpoint:
                self.acts.save(i, h, keep_on_gpu=(i == L))
                h, _ = st.module.forward_train(h, ctx, save=False, qkv_fn=qkv_fn, ln1_weight=ln1)
            else:
                h, saved_all[i] = st.module.forward_train(h, ctx, save=True, qkv_fn=qkv_fn, ln1_weight=ln1)
            self.tracer.end(tok)
            self._check_unit(st, "forward")
            if prefetching:
                # prefetch the next layer(s) into free units
                for j in range(i + 1, min(i + prefetch, L) + 1):
                    if not S[j].resident and S[j].pool.num_free:
                        self._fetch(S[j], with_grad=False, host_leg_only=staged)
            if i == L:
                self._fetch(out, with_grad=True)
            else:
                self._release(st, Event(dev).record())
            if prefetching and i + 1 <= L and not S[i + 1].resident:
                self._fetch(S[i + 1], with_grad=False, host_leg_only=staged)
        if L == 0:
            self._fetch(out, with_grad=True)

        # ---------------- output layer: loss + its backward
        self._wait_loaded(out)
        self._check_unit(out, "forward")
        with self.tracer.span("loss", L + 1):
            loss, dh = out.module.loss_and_grad(h, ctx)
        del h
        if L > 0:
            S[L].bind_device(with_grad=True)
        self._offload_grads(out, step)

        # ---------------- backward through the decoder layers
        for i in range(L, 0, -1):
            st = S[i]
            if i - 1 >= 1:
                self._fetch(S[i - 1], with_grad=True)
                if self.config.enable_activation_checkpoint:
                    self.acts.prefetch(i - 1)
            self._wait_loaded(st)
            self._check_unit(st, "backward")
            tok = self.tracer.begin("bwd", i)
            if self.config.enable_activation_checkpoint:
                h_in = self.acts.get(i)
                _, saved = st.module.forward_train(h_in, ctx, save=True)
                del h_in
            else:
                saved = saved_all.pop(i)
            dh = st.module.backward(saved, dh, ctx, grad_ready=self._grad_ready_hook(st))
            del saved
            self.tracer.end(tok)
            self._offload_grads(st, step)

        # ---------------- embedding backward (weights not needed)
        self._fetch(emb, with_grad=True, need_weights=False)
        self._wait_loaded(emb)
        with self.tracer.span("bwd", 0):
            emb.module.backward_ids(dh, ctx.input_ids)
        del dh
        self._offload_grads(emb, step)
        if self._exact_clip:
            self._apply_exact_clip()
        self.acts.clear()
        self.completed_steps = step
        if self.tracer.enabled:
            self.tracer.step_done(step, {"h2d_bytes": self.h2d_bytes})
        return loss

    def _apply_exact_clip(self) -> None:
        """Every layer's gradient is on the host and measured: combine the
        squared norms over ranks, then start the deferred updates with the
        clip coefficient min(1, clip_grad_norm / (norm + 1e-6)) folded into
        their gradient scale (lowest layer first, as the next forward needs
        it first)."""
        if self._reducer is not None:
            self._reducer.drain()
        self.updates.drain()
        t = torch.tensor([sum(self._clip_parts.values())], dtype=torch.float64, device=self.device)
        if self.world_size > 1 and not self.comm.rank0_optimizer:
            dist.all_reduce(t)
        norm = math.sqrt(float(t.item()))
        coef = min(1.0, self.config.clip_grad_norm / (norm + 1e-6))
        self.last_grad_norm = norm
        deferred, self._deferred, self._clip_parts = self._deferred, {}, {}
        for idx in sorted(deferred):
            fn, g = deferred[idx]
            self.updates.submit(idx, None, lambda fn=fn, g=g: fn(g, coef))

    @torch.no_grad()
    def _inference(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Forward only; returns logits [B, S, V]."""
        ctx = self._make_context(input_ids, None)
        S = self.layer_states
        L = self.num_decoder_layers
        self._fetch(S[0], with_grad=False)
        self._wait_loaded(S[0])
        h = S[0].module.forward_ids(ctx.input_ids)
        self._release(S[0], Event(self.device).record())
        for i in range(1, L + 2):
            st = S[i]
            self._fetch(st, with_grad=False)
            if i + 1 < L + 2 and S[i + 1].pool.num_free:
                self._fetch(S[i + 1], with_grad=False)
            self._wait_loaded(st)
            if i <= L:
                h = st.module(h, ctx)
            else:
                h = st.module.logits(h)
            self._release(st, Event(self.device).record())
        B, T = input_ids.shape
        return h.view(B, T, -1)

    # ------------------------------------------------------------ control
    def wait_for_updates(self) -> None:
        """Block until every scheduled optimizer update (all ranks) landed."""
        self.comm.check()
        if self._reducer is not None:
            self._reducer.drain()
        self.updates.drain()
        for st in self.layer_states:
            self.updates.wait_counter(st.idx, self._update_target(st))

    def update_learning_rate(self, new_lr: float) -> None:
        """Rate for the steps that start from now on.  Updates of earlier
        steps still in flight keep the rate their step ran with (each update
        carries it), so a per-step schedule costs no synchronisation: the
        optimizer tail of one step keeps overlapping the next forward."""
        self.config.lr = new_lr
        if self.layer_optimizer is not None:
            self.layer_optimizer.update_learning_rate(new_lr)

    def clip_grad_norm_(self, max_norm: float) -> torch.Tensor:
        """Global L2 norm of the last step's (averaged) gradients held in host
        memory, summed over ranks' shards.  As in the reference, the fused
        step has already applied the updates by the time this can run, so the
        norm is reported and the held gradients are scaled in place but no
        update is repeated."""
        self.wait_for_updates()
        host = _native.host()
        sq = 0.0
        scale2 = self.comm.grad_scale ** 2
        for st in self.layer_states:
            if st.grad_host is not None and st.grad_host.numel():
                sq += host.sumsq(st.grad_host) * scale2
        t = torch.tensor([sq], dtype=torch.float64, device=self.device)
        if self.world_size > 1 and not self.comm.rank0_optimizer:
            dist.all_reduce(t)
        total = math.sqrt(float(t.item()))
        coef = max_norm / (total + 1e-6)
        if coef < 1:
            for st in self.layer_states:
                if st.grad_host is not None and st.grad_host.numel():
                    host.cast_(st.grad_host, st.grad_host, coef)
        return torch.tensor(total)

    # --------------------------------------------------------- persistence
    def named_master_tensors(self):
        """(HF name, fp32 host view) for every parameter, in model order."""
        out = []
        for st in self.layer_states:
            views = st.layout.views(st.store.read_fp32())
            for e in st.layout.entries:
                if self.generic:
                    name = e.hf_name
                elif st.kind == "embed":
                    name = "model.embed_tokens." + e.name
                elif st.kind == "output":
                    name = ("model." + e.name) if e.name.startswith("norm.") else e.name
                else:
                    name = f"model.layers.{st.idx - 1}.{e.name}"
                out.append((name, views[e.name]))
        return out

    def save_pretrained(self, output_dir: str) -> str:
        """Write an HF-layout checkpoint (config.json + safetensors in
        ``config.dtype``).  Unlike the reference (slide_fsdp.py:705-733) this
        neither converts the live parameters nor stops training."""
        from .utils.checkpoint_io import save_hf_checkpoint

        self.wait_for_updates()
        if self.rank == 0:
            save_hf_checkpoint(output_dir, self._hf_config_dict(),
                               dict(self.named_master_tensors()), self.dtype)
            print(f"Model saved to {output_dir}")
        if self.world_size > 1:
            dist.barrier()
        return output_dir

    def _hf_config_dict(self) -> dict:
        cfg = self.model_config
        return cfg.to_hf_dict() if hasattr(cfg, "to_hf_dict") else cfg.to_dict()

    def save_state(self, directory: str) -> None:
        """fp32 master (rank 0) + this rank's optimizer shards, one file per
        layer index (``layer_<i>.pt`` / ``optim_rank<r>_layer_<i>.pt``) and a
        JSON manifest.  ``load_state`` restores them exactly."""
        self.wait_for_updates()
        os.makedirs(directory, exist_ok=True)
        if self.rank == 0:
            for st in self.layer_states:
                torch.save(st.store.read_fp32().clone(), os.path.join(directory, f"layer_{st.idx}.pt"))
            with open(os.path.join(directory, "manifest.json"), "w") as f:
                json.dump({"world_size": self.world_size, "completed_steps": self.completed_steps,
                           "optimizer_sharding": self.config.optimizer_sharding,
                           "num_layers": self.num_layers, "config": self.config.to_dict(),
                           "model": self._hf_config_dict()}, f, indent=2, default=str)
        if self.layer_optimizer is not None:
            for st in self.layer_states:
                if st.shard[1] > st.shard[0]:
                    sd = self.layer_optimizer.state_dict_for_layer(st.idx)
                    torch.save({"step": sd["step"], "exp_avg": sd["exp_avg"].clone(),
                                "exp_avg_sq": sd["exp_avg_sq"].clone(), "shard": st.shard},
                               os.path.join(directory, f"optim_rank{self.rank}_layer_{st.idx}.pt"))
        if self.world_size > 1:
            dist.barrier()

    def load_state(self, directory: str) -> None:
        """Restore a ``save_state`` directory.  The world size and optimizer
        placement may differ from the saving run's: each rank assembles its
        own shard of every layer's optimizer state from the saved shards that
        overlap it (read through memory maps, so only those bytes are
        read), which lets a run resume on another number of GPUs."""
        self.wait_for_updates()
        with open(os.path.join(directory, "manifest.json")) as f:
            manifest = json.load(f)
        if manifest["num_layers"] != self.num_layers:
            raise ValueError(f"the saved state has {manifest['num_layers']} layers, this model {self.num_layers}")
        if self.rank == 0:
            for st in self.layer_states:
                st.store.write_fp32(torch.load(os.path.join(directory, f"layer_{st.idx}.pt")))
        if self.layer_optimizer is not None:
            saved_world = int(manifest["world_size"])
            for st in self.layer_states:
                if st.shard[1] > st.shard[0]:
                    sd = self._assemble_optimizer_shard(directory, st, saved_world)
                    self.layer_optimizer.load_state_for_layer(st.idx, sd)
        # counters keep counting from here: completed_steps is the number of
        # update rounds already published by this process group
        if self.world_size > 1:
            dist.barrier()

    def _assemble_optimizer_shard(self, directory: str, st: LayerRuntimeState, saved_world: int) -> dict:
        """m, v and step of this rank's range [s, e) of layer ``st`` from the
        saved per-rank files, whatever ranges they cover."""
        s, e = st.shard
        out = None
        covered = 0
        step = None
        for r in range(saved_world):
            path = os.path.join(directory, f"optim_rank{r}_layer_{st.idx}.pt")
            if not os.path.exists(path):
                continue  # that rank owned nothing of this layer
            sd = torch.load(path, mmap=True)
            a, b = (int(x) for x in sd["shard"])
            lo, hi = max(a, s), min(b, e)
            if step is not None and int(sd["step"]) != step:
                raise ValueError(f"layer {st.idx}: saved shards disagree on the step count")
            step = int(sd["step"])
            if hi <= lo:
                continue
            if out is None:
                out = {"exp_avg": torch.empty(e - s, dtype=sd["exp_avg"].dtype),
                       "exp_avg_sq": torch.empty(e - s, dtype=sd["exp_avg_sq"].dtype)}
            for k in ("exp_avg", "exp_avg_sq"):
                out[k][lo - s:hi - s].copy_(sd[k][lo - a:hi - a])
            covered += hi - lo
        if out is None or covered != e - s:
            raise ValueError(f"layer {st.idx}: the saved optimizer shards cover {covered} of the "
                             f"{e - s} elements this rank needs")
        out["step"] = step
        return out

    # --------------------------------------------------------------- misc
    def step_stats(self) -> Dict[str, float]:
        return {"h2d_bytes": float(self.h2d_bytes), "adam_busy_s": self.updates.busy_s,
                "fetch_blocked_s": self.updates.blocked_s,
                "ac_d2h_bytes": float(self.acts.bytes_d2h), "ac_h2d_bytes": float(self.acts.bytes_h2d)}

    def close(self) -> None:
        if getattr(self, "_closed", True):
            return
        self._closed = True
        try:
            self.wait_for_updates()
        except Exception as exc:  # closing still releases everything; say what was lost
            warnings.warn(f"SlideFSDP.close: pending optimizer updates did not complete: {exc}")
        if 1 < self.world_size <= 32:
            # tell the other ranks at their next step that this one is gone
            _native.host().counter_add(self.counters, self._live_base + 32 + self.rank,
                                       self.completed_steps + 1)
        self.updates.close()
        if self._reducer is not None:
            self._reducer.close()
        self.acts.close()
        if self.layer_optimizer is not None:
            self.layer_optimizer.close()
        for st in self.layer_states:
            for e in st.layout.entries:
                e.param.data = torch.empty(0)
                e.param.grad = None
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        self.grad_region.close()
        self.shared.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RankLeftError(RuntimeError):
    """Another rank of the run closed its engine; this rank cannot continue."""


class _SubRegion:
    """A HostRegion view starting at a byte offset (for the cpu_reduce slots)."""

    def __init__(self, region: HostRegion, base: int):
        self.region = region
        self.base = base

    def view(self, dtype, offset_bytes, numel):
        return self.region.view(dtype, self.base + offset_bytes, numel)
