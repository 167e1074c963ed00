"""Host memory for the layer-sliding engine.

``HostRegion`` is one large byte region from which the engine carves typed,
aligned views: the fp32 master, the bf16 shadow, gradient buffers, counters.

* Multi-rank: the region is a file under /dev/shm created sparse by the
  first local rank and mapped MAP_SHARED by every local rank (the role of the
  reference's per-layer ``ssdp_<session>_layer_<i>.bin`` files,
  shared_memory.py:101-156, but one mapping instead of one per layer, no
  zero-fill pass, and page-locked for DMA).
* Single rank: an anonymous private mapping with transparent huge pages.

Both are registered with ``cudaHostRegister`` (portable + mapped) when a GPU
is present, so host<->device copies run at full DMA speed and kernels can
read/write the memory directly (zero-copy).
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch

from .. import _native

ALIGN_BYTES = 4096


def _align(x: int, a: int = ALIGN_BYTES) -> int:
    return (x + a - 1) // a * a


class HostRegion:
    def __init__(self, nbytes: int, shm_path: Optional[str] = None, create: bool = True,
                 pin: bool = False, prefault: bool = False, numa_nodes: Optional[List[int]] = None):
        self.nbytes = max(_align(nbytes), ALIGN_BYTES)
        self.shm_path = shm_path
        self.owner = create
        host = _native.host()
        if shm_path is None:
            self.buf = host.anon_map(self.nbytes, True)
        else:
            self.buf = host.shm_map(shm_path, self.nbytes, create)
        if numa_nodes:
            host.numa_bind(self.buf, list(numa_nodes), "interleave" if len(numa_nodes) > 1 else "preferred")
        if prefault:
            host.prefault(self.buf)
        self.pinned = False
        if pin and torch.cuda.is_available():
            self.pin()
        self._cursor = 0

    # ------------------------------------------------------------ pinning
    def pin(self) -> None:
        if self.pinned:
            return
        # cudaHostRegisterPortable (1) | cudaHostRegisterMapped (2)
        rc = torch.cuda.cudart().cudaHostRegister(self.buf.data_ptr(), self.nbytes, 3)
        if int(rc) != 0:
            raise RuntimeError(f"cudaHostRegister of {self.nbytes} bytes failed with error {int(rc)}")
        self.pinned = True

    def unpin(self) -> None:
        if self.pinned:
            torch.cuda.cudart().cudaHostUnregister(self.buf.data_ptr())
            self.pinned = False

    # -------------------------------------------------------------- views
    def view(self, dtype: torch.dtype, offset_bytes: int, numel: int) -> torch.Tensor:
        es = torch.tensor([], dtype=dtype).element_size()
        end = offset_bytes + numel * es
        if end > self.nbytes:
            raise ValueError(f"view [{offset_bytes}, {end}) exceeds region of {self.nbytes} bytes")
        if offset_bytes % es:
            raise ValueError("misaligned view")
        return self.buf[offset_bytes:end].view(dtype)

    def close(self) -> None:
        if getattr(self, "buf", None) is None:
            return
        self.unpin()  # must precede the unmap, or a later mapping of the same range fails
        self.buf = None
        if self.shm_path is not None and self.owner:
            _native.host().shm_remove(self.shm_path)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RegionPlanner:
    """Bump allocator of aligned sub-ranges, planned before the region
    exists (so every rank computes identical offsets)."""

    def __init__(self, align: int = 256):
        self.align = align
        self.size = 0

    def take(self, nbytes: int) -> int:
        off = _align(self.size, self.align)
        self.size = off + nbytes
        return off
