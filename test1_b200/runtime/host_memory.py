"""Host memory for the layer-sliding engine.

``HostRegion`` is one large byte region from which the engine carves typed,
aligned views: the fp32 master, the bf16 shadow, gradient buffers, counters.

* Multi-rank: the region is a file under /dev/shm created sparse by the
  first local rank and mapped MAP_SHARED by every local rank (the role of the
  reference's per-layer ``ssdp_<session>_layer_<i>.bin`` files,
  shared_memory.py:101-156, but one mapping instead of one per layer, no
  zero-fill pass, and page-locked for DMA).
* Single rank: an anonymous private mapping with transparent huge pages.

On a GPU each rank registers the ranges its own device reads or writes with
``cudaHostRegister`` (mapped, for the current device only), so host<->device
copies run at full DMA speed and kernels can read/write the memory directly
(zero-copy).  The first words of a shared region are a header that the
creating rank writes and every other rank checks (``check_region_header``).
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch

from .. import _native

ALIGN_BYTES = 4096

# Header of a shared region: int64 words [magic, version, then the layout
# fields in REGION_FIELDS order, then a checksum of all previous words].
REGION_MAGIC = 0x4853303032423154  # "T1B200SH" little-endian
REGION_VERSION = 1
REGION_FIELDS = ("region_bytes", "world_size", "num_layers", "total_params", "layout_code")
REGION_HEADER_BYTES = 8 * (3 + len(REGION_FIELDS))


def _align(x: int, a: int = ALIGN_BYTES) -> int:
    return (x + a - 1) // a * a


def mem_available_bytes() -> Optional[int]:
    """The kernel's estimate of memory available to new allocations
    (MemAvailable), or None where /proc/meminfo does not say."""
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return None


def shm_free_bytes(path: str = "/dev/shm") -> Optional[int]:
    """Free space of the shared-memory mount (a file larger than it faults
    with SIGBUS on first touch instead of failing at creation)."""
    try:
        st = os.statvfs(path)
    except OSError:
        return None
    return st.f_bavail * st.f_frsize


def _checksum(words: List[int]) -> int:
    c = 0x9E3779B97F4A7C15
    for w in words:
        c = ((c ^ (w & 0xFFFFFFFFFFFFFFFF)) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return c - (1 << 64) if c >= 1 << 63 else c


def write_region_header(region: "HostRegion", offset: int, fields: dict) -> None:
    """The creating rank stamps the layout it carved the region for, so that
    every rank that maps it later can tell that it expects the same one."""
    words = [REGION_MAGIC, REGION_VERSION] + [int(fields[k]) for k in REGION_FIELDS]
    words.append(_checksum(words))
    region.view(torch.int64, offset, len(words)).copy_(torch.tensor(words, dtype=torch.int64))


def check_region_header(region: "HostRegion", offset: int, fields: dict, rank: int = 0) -> None:
    """Raise a descriptive error unless the header at ``offset`` was written
    for exactly this layout: a region that another program wrote over, a
    damaged header, or local ranks started with different models or
    configurations (each would read the others' bytes as its own tensors)."""
    words = region.view(torch.int64, offset, 3 + len(REGION_FIELDS)).tolist()
    where = region.shm_path or "anonymous region"
    if words[0] != REGION_MAGIC:
        raise RuntimeError(f"rank {rank}: shared host region {where} carries no test1_b200 header "
                           f"(magic {words[0]:#x}); it was overwritten or created by another program")
    if words[-1] != _checksum(words[:-1]):
        raise RuntimeError(f"rank {rank}: the header of shared host region {where} is corrupt (checksum)")
    if words[1] != REGION_VERSION:
        raise RuntimeError(f"rank {rank}: shared host region {where} has header version {words[1]}, "
                           f"expected {REGION_VERSION}")
    for k, got in zip(REGION_FIELDS, words[2:-1]):
        want = int(fields[k])
        if got != want:
            raise RuntimeError(f"rank {rank}: shared host region {where} was laid out for {k} = {got}, "
                               f"this rank expects {want}; every local rank must run the same model "
                               f"and configuration")


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
    PIN_CHUNK = 1 << 30

    def pin(self, ranges: Optional[List[tuple]] = None, strict: bool = True) -> List[tuple]:
        """Page-lock the region for this process's GPU (mapped, not portable:
        each rank drives one device, and registering for every device of the
        node multiplies the DMA mappings by the GPU count), one registration
        per range.  ``ranges`` are (byte offset, size) pairs on page
        boundaries that never share a page -- one per tensor a copy or kernel
        reads, so every transfer lies inside a single registration.  Without
        ranges the region is registered in 1 GiB pieces.

        With ``strict=False`` a range the OS refuses stays pageable (copies
        from it are staged by the driver; kernels cannot map it) and is
        returned; with ``strict=True`` the first refusal raises."""
        if self.pinned:
            return []
        rt = torch.cuda.cudart()
        base = self.buf.data_ptr()
        if ranges is None:
            ranges = [(off, min(self.PIN_CHUNK, self.nbytes - off))
                      for off in range(0, self.nbytes, self.PIN_CHUNK)]
        self._pinned_chunks = []
        self.unpinned_ranges = []
        for off, n in ranges:
            if n <= 0:
                continue
            # cudaHostRegisterMapped (2): pinned and mapped for the current device
            rc = int(rt.cudaHostRegister(base + off, n, 2))
            if rc != 0:
                if strict:
                    for p in self._pinned_chunks:
                        rt.cudaHostUnregister(p)
                    self._pinned_chunks = []
                    raise RuntimeError(f"cudaHostRegister of bytes [{off}, {off + n}) of a {self.nbytes}-byte "
                                       f"host region failed with error {rc}")
                _native.cuda().clear_error()  # the refusal is handled: keep it out of later checks
                self.unpinned_ranges.append((off, n))
                continue
            self._pinned_chunks.append(base + off)
        self.pinned = True
        return list(self.unpinned_ranges)

    def unpin(self) -> None:
        if self.pinned:
            rt = torch.cuda.cudart()
            for p in getattr(self, "_pinned_chunks", []):
                rt.cudaHostUnregister(p)
            self._pinned_chunks = []
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

    def unlink(self) -> None:
        """Remove the shared-memory file while the mappings stay valid: once
        every process that needs the region has mapped it, nothing can leak
        it any more, not even a process that dies without cleaning up."""
        if self.shm_path is not None and self.owner:
            _native.host().shm_remove(self.shm_path)
            self.owner = False

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


class MasterStore:
    """One layer's master weights in host memory.  Layouts:

    * ``split`` -- fp32 stored as a bf16 high plane (which *is* the shadow the
      GPUs load) followed by a 16-bit low plane (see host_kernels.h, kSplit);
    * ``fp32``  -- plain fp32 plus a separate low-precision shadow;
    * ``bf16``  -- bf16 only (the optimizer rounds every update to nearest
      even): the reference's bf16-parameter LayerAdam mode, for models whose
      fp32 master does not fit in host RAM (e.g. 70B on one node).

    All fp32 reads and writes go through this class."""

    def __init__(self, region: "HostRegion", numel: int, master_off: int, split: bool,
                 shadow_dtype: torch.dtype, shadow_off: Optional[int] = None, layout: Optional[str] = None):
        self.numel = numel
        self.layout = layout or ("split" if split else "fp32")
        self.split = self.layout == "split"
        self.lo = None
        if self.layout == "split":
            self.hi = region.view(torch.bfloat16, master_off, numel)
            self.lo = region.view(torch.int16, master_off + 2 * numel, numel)
            self.f32 = None
            self.shadow = self.hi
        elif self.layout == "bf16":
            self.hi = region.view(torch.bfloat16, master_off, numel)
            self.f32 = None
            self.shadow = self.hi
        else:
            self.f32 = region.view(torch.float32, master_off, numel)
            self.hi = None
            if shadow_dtype == torch.float32 or shadow_off is None:
                self.shadow = self.f32
            else:
                self.shadow = region.view(shadow_dtype, shadow_off, numel)

    @staticmethod
    def bytes_needed(numel: int, split: bool, shadow: bool, layout: Optional[str] = None) -> tuple:
        """(master bytes, shadow bytes) to plan for one layer."""
        layout = layout or ("split" if split else "fp32")
        if layout == "bf16":
            return 2 * numel, 0
        return 4 * numel, (0 if layout == "split" or not shadow else 2 * numel)

    @property
    def bind_tensor(self) -> torch.Tensor:
        """Flat tensor the offloaded module parameters point into."""
        return self.hi if self.f32 is None else self.f32

    def read_fp32(self, s: int = 0, e: Optional[int] = None, out: Optional[torch.Tensor] = None):
        e = self.numel if e is None else e
        if self.layout == "fp32":
            return self.f32[s:e] if out is None else out.copy_(self.f32[s:e])
        if self.layout == "bf16":
            return self.hi[s:e].float() if out is None else out.copy_(self.hi[s:e])
        out = torch.empty(e - s, dtype=torch.float32) if out is None else out
        _native.host().split_to_f32(self.hi[s:e], self.lo[s:e], out)
        return out

    def write_fp32(self, src: torch.Tensor, s: int = 0) -> None:
        e = s + src.numel()
        src = src.reshape(-1).float().contiguous()
        if self.layout == "split":
            _native.host().f32_to_split(src, self.hi[s:e], self.lo[s:e])
        elif self.layout == "bf16":
            _native.host().cast_(self.hi[s:e], src, 1.0)
        else:
            self.f32[s:e].copy_(src)
            if self.shadow is not self.f32:
                _native.host().cast_(self.shadow[s:e], self.f32[s:e], 1.0)

    def optim_slice(self, s: int, e: int):
        if self.layout == "split":
            return self.hi[s:e], self.lo[s:e]
        return self.hi[s:e] if self.layout == "bf16" else self.f32[s:e]
