"""GPU buffer pool and per-layer runtime state of the sliding engine.

Counterparts of the reference's ``LayerBufferPool`` and ``LayerRuntimeState``
(layer_state.py:28-467), redesigned:

* Pool units are reused under CUDA-event ordering instead of host-side
  ``synchronize`` calls: each unit carries the event after which the GPU is
  done with its previous occupant, and every copy into the unit waits on it.
  The host never blocks to recycle a unit.
* ``acquire`` fails loudly on exhaustion (the reference pops from an empty
  deque, layer_state.py:78-91).
* Units are sized by the largest *decoder* layer; the embedding and the
  output layer (norm + lm_head, 2.4x a Llama-3.1-8B decoder layer) share one
  dedicated large unit, whose use never overlaps (embedding forward happens
  first, output layer last, and the embedding backward needs no weights).
* Flat layout: a layer's parameters are concatenated in ``named_parameters``
  order (the reference's order, layer_state.py:241-264); each layer's region
  starts on a 256-byte boundary; shard boundaries are multiples of 64
  elements (the reference uses unaligned ``ceil(P/N)`` chunks,
  distributed_sync.py:84-96).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .device import Event

SHARD_ALIGN = 64  # elements


def shard_bounds(numel: int, world: int, rank: int, align: int = SHARD_ALIGN) -> Tuple[int, int]:
    per = -(-numel // world)
    per = -(-per // align) * align
    start = min(rank * per, numel)
    return start, min(start + per, numel)


def shard_size(numel: int, world: int, align: int = SHARD_ALIGN) -> int:
    per = -(-numel // world)
    return -(-per // align) * align


@dataclass
class ParamEntry:
    name: str
    param: nn.Parameter
    shape: torch.Size
    numel: int
    offset: int  # element offset inside the layer's flat buffer
    hf_name: str = ""  # full HF parameter name (generic-architecture path)


@dataclass
class LayerLayout:
    idx: int
    kind: str  # "embed" | "decoder" | "output"
    entries: List[ParamEntry]
    numel: int
    master_off: int = 0  # byte offsets into the host regions
    shadow_off: int = 0

    def views(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {e.name: flat[e.offset:e.offset + e.numel].view(e.shape) for e in self.entries}


def build_layout(idx: int, kind: str, module: nn.Module) -> LayerLayout:
    entries, off = [], 0
    seen = set()
    for name, p in module.named_parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        entries.append(ParamEntry(name, p, p.shape, p.numel(), off))
        off += p.numel()
    return LayerLayout(idx=idx, kind=kind, entries=entries, numel=off)


def _replace_param(root: nn.Module, dotted: str, new: nn.Parameter) -> None:
    *path, leaf = dotted.split(".")
    mod = root
    for part in path:
        mod = getattr(mod, part)
    setattr(mod, leaf, new)


class PoolUnit:
    def __init__(self, uid: int, param: torch.Tensor, grad: torch.Tensor):
        self.uid = uid
        self.param = param
        self.grad = grad
        self.free_event: Optional[Event] = None  # GPU done with the previous occupant
        self.owner: Optional[int] = None


class LayerBufferPool:
    """A fixed set of GPU units, each a flat ``param`` and ``grad`` buffer of
    ``capacity`` elements."""

    def __init__(self, capacity: int, dtype: torch.dtype, device: torch.device, pool_size: int,
                 allocator=None, name: str = "pool"):
        self.capacity = capacity
        self.dtype = dtype
        self.device = device
        self.pool_size = pool_size
        self.name = name
        alloc = allocator or (lambda n: torch.empty(n, dtype=dtype, device=device))
        self.units = [PoolUnit(i, alloc(capacity), alloc(capacity)) for i in range(pool_size)]
        self._free: List[PoolUnit] = list(self.units)

    def acquire(self, layer_idx: int) -> PoolUnit:
        if not self._free:
            owners = [u.owner for u in self.units]
            raise RuntimeError(f"{self.name}: all {self.pool_size} units are in use (owners {owners}); "
                               f"cannot load layer {layer_idx}")
        u = self._free.pop(0)
        u.owner = layer_idx
        return u

    def release(self, unit: PoolUnit, free_event: Optional[Event]) -> None:
        if unit in self._free:
            raise RuntimeError(f"{self.name}: unit {unit.uid} released twice")
        unit.owner = None
        unit.free_event = free_event
        self._free.append(unit)

    @property
    def num_free(self) -> int:
        return len(self._free)


class LayerRuntimeState:
    """Host/GPU bookkeeping of one layer: where its master, shadow and
    gradient live, which pool unit holds it, and the events of its last GPU
    operations."""

    def __init__(self, layout: LayerLayout, module: nn.Module, master: torch.Tensor,
                 shadow: torch.Tensor, grad_host: Optional[torch.Tensor],
                 shard: Tuple[int, int]):
        self.layout = layout
        self.idx = layout.idx
        self.kind = layout.kind
        self.module = module
        self.numel = layout.numel
        self.master = master            # fp32 [numel] host (shared across ranks)
        self.shadow = shadow            # bf16 [numel] host, written by the optimizer
        self.grad_host = grad_host      # host gradient for this rank's update range
        self.shard = shard              # (start, end) this rank updates
        self.unit: Optional[PoolUnit] = None
        self.pool: Optional[LayerBufferPool] = None
        self.loaded: Optional[Event] = None
        self._host_views = layout.views(master)

    # parameter rebinding ------------------------------------------------
    def bind_device(self, with_grad: bool) -> None:
        assert self.unit is not None
        pv = self.layout.views(self.unit.param)
        gv = self.layout.views(self.unit.grad) if with_grad else None
        for e in self.layout.entries:
            e.param.data = pv[e.name]
            e.param.grad = gv[e.name] if with_grad else None

    def bind_host(self) -> None:
        for e in self.layout.entries:
            if e.param.is_meta:
                # a deferred-initialisation model: swap in a real Parameter
                # whose storage is the host master view
                new = nn.Parameter(self._host_views[e.name], requires_grad=e.param.requires_grad)
                _replace_param(getattr(self.module, "params_root", self.module), e.name, new)
                e.param = new
            else:
                e.param.data = self._host_views[e.name]
            e.param.grad = None

    @property
    def resident(self) -> bool:
        return self.unit is not None
