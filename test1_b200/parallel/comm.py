"""Parameter-fetch and gradient-sync strategies of the sliding engine.

Counterpart of the reference's DistributedSync / NoOpSync
(distributed_sync.py:21-377).  The four modes keep their meaning:

  param_transfer_mode
    full   every rank copies the whole layer host->device
    shard  every rank copies 1/N of the layer, then an all-gather rebuilds it
  grad_sync_mode
    gpu_reduce  gradients are reduced on the GPUs, then copied to the host
    cpu_reduce  every rank copies its full gradient to the host; the ranks
                reduce on the CPU

Differences from the reference (each checked by tests against a
single-process oracle):

  * optimizer work is sharded: rank r updates elements shard_bounds(P, N, r)
    of every layer, so ``gpu_reduce`` is a reduce-scatter (each rank copies
    only its 1/N shard to the host) and ``cpu_reduce`` is a shared-memory
    reduce-scatter (each rank sums its slice across all ranks' slots).  The
    reference funnels everything to rank 0 (``reduce(dst=0)``,
    distributed_sync.py:242-300); ``optimizer_sharding="rank0"`` keeps that
    placement.
  * the 1/N averaging is folded into the optimizer's gradient scale (no extra
    pass over the gradient);
  * all collectives are issued by the main thread in program order, on two
    process groups (parameters and gradients) so an all-gather for layer i-1
    and a reduce-scatter for layer i can overlap (the reference issues NCCL
    from a worker thread and barriers from another, distributed_sync.py /
    layer_state.py:432);
  * shard mode gathers in place into the pool unit (no per-call allocation of
    N temporaries and N copy-backs, distributed_sync.py:137-158).

The fused NVLink kernels (``parallel.fused``) replace the all-gather and the
reduce-scatter + device-to-host copy when ``config.fused_comm`` is set and
the ranks are GPUs of one node.
"""
from __future__ import annotations

import os
import threading
import time
from datetime import timedelta
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import _native
from ..runtime.device import Event, Stream
from ..runtime.layer_state import LayerRuntimeState, shard_bounds, shard_size


class CommStrategy:
    """Base: single rank (the reference's NoOpSync)."""

    name = "local"

    def __init__(self, config, device: torch.device, rank: int = 0, world: int = 1):
        self.config = config
        self.device = device
        self.rank = rank
        self.world = world
        self.param_mode = config.param_transfer_mode
        self.grad_mode = config.grad_sync_mode
        self.rank0_optimizer = config.optimizer_sharding == "rank0" and world > 1

    # sizes ---------------------------------------------------------------
    def unit_capacity(self, numel: int) -> int:
        return numel

    def update_range(self, numel: int):
        """Element range of a layer that this rank's optimizer updates."""
        if self.world == 1:
            return 0, numel
        if self.rank0_optimizer:
            return (0, numel) if self.rank == 0 else (0, 0)
        return shard_bounds(numel, self.world, self.rank)

    def updaters_for(self, numel: int) -> int:
        """How many ranks publish an update of a layer of ``numel`` elements
        (ranks whose update range is empty do not)."""
        if self.world == 1 or self.rank0_optimizer:
            return 1
        ss = shard_size(numel, self.world)
        return max(1, -(-numel // ss))

    @property
    def grad_scale(self) -> float:
        return 1.0 / self.world

    # operations ----------------------------------------------------------
    def fetch_params(self, st: LayerRuntimeState, dst: torch.Tensor, stream: Stream) -> None:
        with stream.ctx():
            dst[: st.numel].copy_(st.shadow, non_blocking=True)

    def host_read_views(self, st: LayerRuntimeState) -> list:
        """The host tensors this rank's GPU reads when ``fetch_params`` loads
        layer ``st`` (the engine page-locks exactly these)."""
        return [st.shadow]

    def h2d_bytes(self, st: LayerRuntimeState, element_size: int) -> int:
        """Bytes one ``fetch_params`` of ``st`` moves over this rank's host link."""
        return st.numel * element_size

    def fetch_host_leg(self, st: LayerRuntimeState, dst: torch.Tensor, stream: Stream) -> bool:
        """Only the host-to-device part of a shard fetch (strategies that
        stage it); False when the strategy has none."""
        return False

    def sync_grads(self, st: LayerRuntimeState, src: torch.Tensor, stream: Stream) -> None:
        """Enqueue on ``stream`` everything that moves this rank's share of
        the layer gradient into ``st.grad_host``."""
        if st.grad_host is None or st.grad_host.numel() == 0:
            return
        with stream.ctx():
            st.grad_host.copy_(src[: st.numel], non_blocking=True)

    def host_reduce(self, st: LayerRuntimeState, step: int) -> Optional[torch.Tensor]:
        """Host-side part of the gradient reduction, run on the reducer
        thread once this rank's device-to-host copy finished.  Returns the
        gradient tensor the optimizer consumes."""
        return st.grad_host

    def barrier(self) -> None:
        pass

    def allocator(self, dtype: torch.dtype):
        """Allocation function for pool buffers (None: plain device memory)."""
        return None

    def check(self) -> None:
        """Raise if an asynchronous communication kernel reported an error."""

    def close(self) -> None:
        pass


class CollectiveComm(CommStrategy):
    """NCCL (GPU) / gloo (CPU) collectives: the baseline multi-rank path."""

    name = "collective"

    def __init__(self, config, device: torch.device, rank: int, world: int,
                 cpu_slots: Optional["CpuReduceSlots"] = None):
        super().__init__(config, device, rank, world)
        backend = "nccl" if device.type == "cuda" else "gloo"
        # Separate communicators so parameter gathers and gradient reductions
        # of neighbouring layers can run concurrently.  Their set-up and
        # collectives wait for a peer at most host_wait_timeout_s (the default
        # of new_group would be 30 minutes when a peer never arrives).
        tmo = timedelta(seconds=max(1.0, float(getattr(config, "host_wait_timeout_s", 600.0))))
        self.param_group = (dist.new_group(backend=backend, timeout=tmo)
                            if self.param_mode == "shard" else None)
        self.grad_group = dist.new_group(backend=backend, timeout=tmo)
        self.cpu_slots = cpu_slots
        self._shard_bufs = {}

    def unit_capacity(self, numel: int) -> int:
        if self.param_mode == "shard" or (self.grad_mode == "gpu_reduce" and not self.rank0_optimizer):
            return self.world * shard_size(numel, self.world)
        return numel

    def host_read_views(self, st: LayerRuntimeState) -> list:
        if self.param_mode == "full":
            return super().host_read_views(st)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        return [st.shadow[s:e]] if e > s else []

    def h2d_bytes(self, st: LayerRuntimeState, element_size: int) -> int:
        if self.param_mode == "full":
            return super().h2d_bytes(st, element_size)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        return max(0, e - s) * element_size

    def fetch_params(self, st: LayerRuntimeState, dst: torch.Tensor, stream: Stream) -> None:
        if self.param_mode == "full":
            return super().fetch_params(st, dst, stream)
        ss = shard_size(st.numel, self.world)
        s, e = shard_bounds(st.numel, self.world, self.rank)
        with stream.ctx():
            mine = dst[self.rank * ss:(self.rank + 1) * ss]
            if e > s:
                mine[: e - s].copy_(st.shadow[s:e], non_blocking=True)
            dist.all_gather_into_tensor(dst[: self.world * ss], mine, group=self.param_group)

    def _shard_buf(self, n: int, dtype) -> torch.Tensor:
        key = (n, dtype)
        if key not in self._shard_bufs:
            self._shard_bufs[key] = torch.empty(n, dtype=dtype, device=self.device)
        return self._shard_bufs[key]

    def sync_grads(self, st: LayerRuntimeState, src: torch.Tensor, stream: Stream) -> None:
        P = st.numel
        with stream.ctx():
            if self.grad_mode == "cpu_reduce":
                slot = self.cpu_slots.acquire_for_write(st.idx)
                slot[:P].copy_(src[:P], non_blocking=True)
                return
            if self.rank0_optimizer:
                dist.reduce(src[:P], dst=0, group=self.grad_group)
                if self.rank == 0:
                    st.grad_host.copy_(src[:P], non_blocking=True)
                return
            ss = shard_size(P, self.world)
            s, e = shard_bounds(P, self.world, self.rank)
            out = self._shard_buf(ss, src.dtype)
            dist.reduce_scatter_tensor(out, src[: self.world * ss], group=self.grad_group)
            if e > s:
                st.grad_host.copy_(out[: e - s], non_blocking=True)

    def host_reduce(self, st: LayerRuntimeState, step: int) -> Optional[torch.Tensor]:
        if self.grad_mode != "cpu_reduce":
            return st.grad_host
        return self.cpu_slots.reduce(st, step, self.update_range(st.numel))

    def barrier(self) -> None:
        dist.barrier(group=self.grad_group)


class CpuReduceSlots:
    """Shared-memory gradient slots for ``cpu_reduce``.

    A ring of ``n_slots`` slots, each holding one bf16 gradient per rank.
    Layer i uses slot i % n_slots.  Protocol per layer and step (all counters
    monotonic, in the shared counter region):

      written[i]  += 1 by every rank once its device-to-host copy landed
      consumed[i] += 1 by every rank once it summed its slice of slot i

    A rank reuses a slot for layer i only after every rank consumed the
    slot's previous layer (i + n_slots) of the same step.  This replaces the
    reference's Gloo ``reduce`` to rank 0 (distributed_sync.py:283-300).
    """

    def __init__(self, region, counters: torch.Tensor, counter_base: int, n_layers: int,
                 capacity: int, rank: int, world: int, n_slots: int, timeout_s: float = 600.0,
                 dtype: torch.dtype = torch.bfloat16):
        self.region = region
        self.counters = counters
        self.base = counter_base
        self.n_layers = n_layers
        self.capacity = capacity
        self.rank = rank
        self.world = world
        self.n_slots = n_slots
        self.timeout_s = timeout_s
        self.dtype = dtype
        self.es = torch.tensor([], dtype=dtype).element_size()
        self._host = _native.host()
        self.step = 0

    @staticmethod
    def region_bytes(capacity: int, world: int, n_slots: int, es: int = 2) -> int:
        return n_slots * world * capacity * es

    def _slot(self, layer: int, rank: int) -> torch.Tensor:
        s = layer % self.n_slots
        off = ((s * self.world) + rank) * self.capacity * self.es
        return self.region.view(self.dtype, off, self.capacity)

    def _written(self, layer):
        return self.base + layer

    def _consumed(self, layer):
        return self.base + self.n_layers + layer

    def _wait(self, idx: int, target: int, what: str) -> None:
        if not self._host.counter_wait_geq(self.counters, idx, target, self.timeout_s):
            raise TimeoutError(f"cpu_reduce: {what} (counter {idx} < {target}); a peer rank may have died")

    def acquire_for_write(self, layer: int) -> torch.Tensor:
        """Called by the main thread before the device-to-host copy of layer
        ``layer``'s gradient in step ``self.step``."""
        prev = layer + self.n_slots
        if prev < self.n_layers:
            self._wait(self._consumed(prev), self.world * self.step, f"slot of layer {prev} not consumed")
        elif self.step > 1:
            # previous occupant is this same layer... from the previous step
            pass
        # the slot's previous user in the *previous* step is covered because
        # every layer of a step is consumed before the step ends.
        return self._slot(layer, self.rank)

    def reduce(self, st: LayerRuntimeState, step: int, rng) -> Optional[torch.Tensor]:
        """Publish this rank's slot, wait for all ranks, sum our range."""
        layer = st.idx
        self._host.counter_add(self.counters, self._written(layer), 1)
        self._wait(self._written(layer), self.world * step, f"gradients of layer {layer} not written")
        s, e = rng
        out = None
        if e > s:
            srcs = [self._slot(layer, r)[s:e] for r in range(self.world)]  # slots hold [0, P)
            out = st.grad_host
            self._host.sum_slots_(out, srcs, 1.0)
        self._host.counter_add(self.counters, self._consumed(layer), 1)
        return out


def make_comm(config, device: torch.device, rank: int, world: int, cpu_slots=None) -> CommStrategy:
    if world == 1:
        return CommStrategy(config, device, 0, 1)
    if getattr(config, "fused_comm", False):
        from .fused import FusedComm, symmetric_memory_available

        if symmetric_memory_available(device, world):
            return FusedComm(config, device, rank, world, cpu_slots)
    return CollectiveComm(config, device, rank, world, cpu_slots)
