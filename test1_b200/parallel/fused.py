"""Fused NVLink communication for the sliding engine (one process per GPU,
all GPUs of one node).  It replaces the reference's shard all-gather
(distributed_sync.py:118-158) and gpu_reduce gradient reduction
(distributed_sync.py:242-300, reduce to rank 0 + D2H) with kernels that move
the data over peer memory themselves.

The pool units live in symmetric memory (``torch.distributed._symmetric_memory``:
one allocation per buffer, mapped into every rank, plus a per-buffer signal
pad).  Two sm_100a kernels (``csrc/cuda/fused_comm.cu``) replace NCCL on the
engine's hot paths:

  gpu_reduce   ``fused_rs_d2h``: reduce-scatter of the layer gradient over
               NVLink (P2P loads from every peer's unit), scaled by 1/N,
               rounded to bf16 and stored directly into this rank's
               page-locked host gradient shard (zero-copy).
  shard        staged (default, ``shard_source="shadow"``): the copy engine
               moves this rank's shard of the layer's bf16 copy (the high
               plane of the split master, 2 B/param) into its own unit, then
               ``fused_shard_gather`` broadcasts it into every peer's unit
               (P2P stores over NVLink) on a few CTAs, one layer ahead of
               use, like full mode's prefetch; or the broadcast runs inside
               the layer's QKV GEMM (``fused_ag_qkv``, ``fuse_gather_qkv``).
               ``shard_source="master"``: the kernels read the fp32 master
               (both planes, 4 B/param) from page-locked host memory
               themselves and round it to bf16 on the GPU.

Buffers keep a per-buffer epoch counter (identical on every rank because the
schedule is); kernels signal and wait on it with bounded waits and report
expiry through an error word that ``check()`` turns into an exception.
cpu_reduce keeps the shared-memory slot reduction of ``CollectiveComm``.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.distributed as dist

from .. import _native
from ..runtime.device import Stream
from ..runtime.layer_state import LayerRuntimeState, shard_bounds
from .comm import CollectiveComm


def symmetric_memory_available(device: torch.device, world: int) -> bool:
    if device.type != "cuda" or world < 2 or world > 8:
        return False
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except Exception:
        return False
    return True


class SymmetricBuffer:
    """A symmetric allocation plus what the kernels need: peer base
    pointers, peer signal pads, an epoch counter and a completion counter."""

    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device, group):
        import torch.distributed._symmetric_memory as symm_mem

        self.tensor = symm_mem.empty(numel, dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.tensor, group)
        self.ptrs = torch.tensor(list(self.handle.buffer_ptrs), dtype=torch.int64)
        self.sigs = torch.tensor(list(self.handle.signal_pad_ptrs), dtype=torch.int64)
        self.epoch = 0
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.ag_counters = torch.zeros(65, dtype=torch.int32, device=device)
        world = len(self.handle.buffer_ptrs)
        need = (2 * world + 64 * world) * 4
        if self.handle.signal_pad_size < need:
            raise RuntimeError(f"symmetric-memory signal pad of {self.handle.signal_pad_size} bytes is "
                               f"smaller than the {need} bytes the fused kernels use")

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch


class FusedComm(CollectiveComm):
    name = "fused-nvlink"

    def __init__(self, config, device: torch.device, rank: int, world: int, cpu_slots=None):
        super().__init__(config, device, rank, world, cpu_slots)
        import torch.distributed._symmetric_memory as symm_mem

        self.group = dist.group.WORLD
        try:
            symm_mem.enable_symm_mem_for_group(self.group.group_name)
        except Exception:
            pass
        self._bufs: Dict[int, SymmetricBuffer] = {}
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.fused_grads = self.grad_mode == "gpu_reduce" and not self.rank0_optimizer
        self.fused_params = self.param_mode == "shard"
        src = getattr(config, "shard_source", "shadow")
        self.shard_source = src if src in ("master", "shadow") else "shadow"
        self.gather_ctas = int(getattr(config, "shard_gather_ctas", 64))
        self._peer_tail = None  # completion event of the last peer-waiting kernel

    def disable_fused(self, params: bool, grads: bool) -> None:
        """Fall back to the NCCL path for parameter gathers and/or gradient
        reductions (every rank must make the same call, before the pools are
        allocated): used when host memory a fused kernel must map could not
        be page-locked."""
        if params:
            self.fused_params = False
        if grads:
            self.fused_grads = False

    # pool allocation -----------------------------------------------------
    def unit_capacity(self, numel: int) -> int:
        if self.fused_grads or self.fused_params:
            return numel
        return super().unit_capacity(numel)

    def allocator(self, dtype: torch.dtype):
        def alloc(n: int) -> torch.Tensor:
            b = SymmetricBuffer(n, dtype, self.device, self.group)
            self._bufs[b.tensor.data_ptr()] = b
            return b.tensor
        return alloc

    def _buf(self, t: torch.Tensor) -> SymmetricBuffer:
        b = self._bufs.get(t.data_ptr())
        if b is None:
            raise RuntimeError("fused communication needs pool units allocated in symmetric memory")
        return b

    @property
    def grad_scale(self) -> float:
        # the fused reduce-scatter already multiplies by 1/N
        return 1.0 if self.fused_grads else 1.0 / self.world

    # ordering of the kernels that wait on peer GPUs ----------------------
    def _peer_launch(self, stream: Optional[torch.cuda.Stream] = None):
        """Context for one launch of a kernel that waits on peer GPUs (a
        gather, a reduce-scatter or the fused QKV GEMM): it starts only after
        the previous such kernel of this rank completed, on whatever stream.
        Every rank launches them in the same program order, so each GPU then
        runs them in that order and the k-th kernel of one rank always meets
        the k-th of the others.  Without it, two of them on different streams
        can start in different orders on two GPUs; one that holds every SM
        (the fused QKV GEMM) keeps the other from starting, and each rank
        waits for a peer kernel that cannot run (seen as expired peer waits,
        errors 211/212, in a 2-GPU shard-mode run)."""
        fc = self

        class _Ctx:
            def __enter__(self_):
                s = stream if stream is not None else torch.cuda.current_stream(fc.device)
                self_.s = s
                self_.cm = torch.cuda.stream(s)
                self_.cm.__enter__()
                if fc._peer_tail is not None:
                    s.wait_event(fc._peer_tail)
                return s

            def __exit__(self_, *exc):
                ev = torch.cuda.Event()
                ev.record(self_.s)
                fc._peer_tail = ev
                return self_.cm.__exit__(*exc)

        return _Ctx()

    # operations ----------------------------------------------------------
    @property
    def staged(self) -> bool:
        """Shard fetches move the host leg with the copy engine (bf16 copy)."""
        return self.fused_params and self.shard_source == "shadow"

    def fetch_host_leg(self, st: LayerRuntimeState, dst: torch.Tensor, stream: Stream) -> bool:
        """Staged shard mode: enqueue on ``stream`` the copy-engine transfer of
        this rank's shard of the layer's bf16 copy into its own unit.  Returns
        False (nothing enqueued) when shard fetches are not staged."""
        if not self.staged:
            return False
        s, e = shard_bounds(st.numel, self.world, self.rank)
        if e > s:
            with stream.ctx():
                dst[s:e].copy_(st.shadow[s:e], non_blocking=True)
        return True

    def fetch_params(self, st: LayerRuntimeState, dst: torch.Tensor, stream: Stream) -> None:
        if not self.fused_params:
            return super().fetch_params(st, dst, stream)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        b = self._buf(dst)
        if self.fetch_host_leg(st, dst, stream):
            # NVLink leg on a few CTAs: the shard, now in this rank's unit,
            # into every peer's
            with self._peer_launch(stream.s):
                _native.cuda().fused_shard_gather(b.ptrs, b.sigs, self.rank, self.world, s, e - s,
                                                  dst[s:e] if e > s else dst[:0], None, b.next_epoch(),
                                                  b.counter, self.err, self.gather_ctas)
            return
        src, lo = self._gather_src(st, s, e)
        with self._peer_launch(stream.s):
            _native.cuda().fused_shard_gather(b.ptrs, b.sigs, self.rank, self.world, s, e - s,
                                              src, lo, b.next_epoch(), b.counter, self.err)

    def h2d_bytes(self, st: LayerRuntimeState, element_size: int) -> int:
        """Bytes one parameter fetch of ``st`` moves over this rank's host link."""
        if not self.fused_params:
            return super().h2d_bytes(st, element_size)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        if self.staged:
            return 2 * max(0, e - s)
        src, lo = self._gather_src(st, s, e)
        return max(0, e - s) * (4 if (lo is not None or src.element_size() == 4) else 2)

    def host_read_views(self, st: LayerRuntimeState) -> list:
        if not self.fused_params:
            return super().host_read_views(st)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        if e <= s:
            return []
        if self.staged:
            return [st.shadow[s:e]]
        return [t for t in self._gather_src(st, s, e) if t is not None]

    def sync_grads(self, st: LayerRuntimeState, src: torch.Tensor, stream: Stream) -> None:
        if not self.fused_grads:
            return super().sync_grads(st, src, stream)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        b = self._buf(src)
        out = st.grad_host if st.grad_host is not None else torch.empty(0, dtype=src.dtype)
        with self._peer_launch(stream.s):
            _native.cuda().fused_rs_d2h(b.ptrs, b.sigs, self.rank, self.world, s, e - s, out,
                                        1.0 / self.world, b.next_epoch(), b.counter, self.err)

    def sync_grads_range(self, st: LayerRuntimeState, src: torch.Tensor, stream: Stream,
                         lo: int, hi: int) -> None:
        """Reduce-scatter elements [lo, hi) of the layer gradient as soon as
        they are final (one launch per parameter tensor, in backward order),
        so the NVLink pull and the host store overlap the rest of the
        layer's backward.  Every rank launches for every range, also when
        its shard misses the range (that launch only handshakes)."""
        s, e = shard_bounds(st.numel, self.world, self.rank)
        a, b_ = max(lo, s), min(hi, e)
        n = max(0, b_ - a)
        buf = self._buf(src)
        if n and st.grad_host is not None:
            out = st.grad_host[a - s: a - s + n]
        else:
            out, a, n = torch.empty(0, dtype=src.dtype), lo, 0
        with self._peer_launch(stream.s):
            _native.cuda().fused_rs_d2h(buf.ptrs, buf.sigs, self.rank, self.world, a, n, out,
                                        1.0 / self.world, buf.next_epoch(), buf.counter, self.err)

    @property
    def grads_by_range(self) -> bool:
        return self.fused_grads

    # shard-mode forward: layer fetch fused with the QKV projection -----
    def can_fuse_qkv(self, st: LayerRuntimeState) -> bool:
        return self.fused_params and st.kind == "decoder" and self.device.type == "cuda"

    def shard_table(self, numel: int) -> torch.Tensor:
        key = numel
        t = self._shard_tables.get(key) if hasattr(self, "_shard_tables") else None
        if t is None:
            if not hasattr(self, "_shard_tables"):
                self._shard_tables = {}
            t = torch.tensor([list(shard_bounds(numel, self.world, q)) for q in range(self.world)],
                             dtype=torch.int64)
            self._shard_tables[key] = t
        return t

    def ag_qkv(self, st: LayerRuntimeState, x1: torch.Tensor, n_rows: int, rope=None) -> torch.Tensor:
        """Gather layer ``st`` into every rank's unit and return x1 @ W_qkv^T
        (one kernel, on the current stream), with the rotary embedding of the
        q and k heads applied when ``rope`` = (cos, sin, seq_len, n_q, n_kv,
        head_dim) is given -- in the kernel's epilogue when it can, else by
        the RoPE kernel after it.  Staged: the shard already sits in this
        rank's unit (``fetch_host_leg``), so the kernel's gather warps read it
        from local memory and only push it to the peers."""
        s, e = shard_bounds(st.numel, self.world, self.rank)
        b = self._buf(st.unit.param)
        if self.staged:
            src, lo = st.unit.param[s:e], None
        else:
            src, lo = self._gather_src(st, s, e)
        out = torch.empty(x1.shape[0], n_rows, dtype=x1.dtype, device=x1.device)
        from ..ops import native

        fuse_rope = rope is not None and native.rope_fusable(rope[5])
        cos, sin, S, n_rot = (None, None, 1, 0) if not fuse_rope else (rope[0], rope[1], rope[2],
                                                                      (rope[3] + rope[4]) * rope[5])
        with self._peer_launch():
            _native.cuda().fused_ag_qkv(x1, b.tensor, n_rows, out, b.ptrs, b.sigs,
                                        self.shard_table(st.numel), self.rank, self.world, src, lo,
                                        b.next_epoch(), b.ag_counters, cos, sin, S, n_rot)
        if rope is not None and not fuse_rope:
            cos, sin, S, n_q, n_kv, D = rope
            native.rope_qkv_(out, n_q, n_kv, D, cos, sin, S)
        return out

    def _gather_src(self, st: LayerRuntimeState, s: int, e: int):
        """(tensor, low plane or None) the shard fetch reads from host
        memory: the fp32 master -- plain, or both planes of a split master --
        cast to bf16 (nearest even) on the GPU; or the bf16 copy."""
        store = getattr(st, "store", None)
        if self.shard_source == "master" and store is not None:
            if store.split:
                return store.hi[s:e], store.lo[s:e]
            if store.f32 is not None:
                return store.f32[s:e], None
        return st.shadow[s:e], None

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"fused NVLink kernel reported error {code} (a bounded cross-GPU wait "
                               f"expired: a peer rank stalled or died)")
