"""SlidingCheckpoint: offload the tensors saved by a checkpointed layer to
host memory (or NVMe) during the forward pass and bring them back one layer
ahead during the backward pass.

Public constructor and behaviour of the reference's class
(sliding_checkpoint.py:11-204): a ``torch.autograd.graph.saved_tensors_hooks``
context used around ``torch.utils.checkpoint(..., use_reentrant=False)`` of
decoder layer ``layer_idx`` (1-based); the k-th saved tensor of layer i goes
to the preallocated pinned slot ``layer_tensors[i-1][k]``; the last layer
keeps its tensors on the GPU; on the first unpack of layer i the slots of
layer i-1 are copied back to the GPU on a side stream.

Differences from the reference (sliding_checkpoint.py:11-202), each fixing one of its defects:
  * the GPU tensor being offloaded is kept alive (``record_stream``) until
    its copy on the side stream completed;
  * prefetched buffers are keyed by layer, not a global FIFO, so an
    unexpected order can never hand a layer another layer's tensors;
  * ``gds_offload=True`` works without kvikio: slots are written to / read
    from files under ``file_paths`` by a background thread;
  * with ``layer_tensors=None`` (the reference asserts) tensors stay on the
    GPU;
  * on a CPU-only run the hooks pass tensors through.

The SlideFSDP engine itself checkpoints one tensor per layer through
``runtime.activations.ActivationStore``; this class is the general-purpose
hook for user code built around ``torch.utils.checkpoint``.
"""
from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Dict, List, Optional, Tuple

import torch
from torch.autograd.graph import saved_tensors_hooks

_side_stream: Dict[int, "torch.cuda.Stream"] = {}
_prefetched: Dict[int, Tuple[List[torch.Tensor], Any]] = {}
_lock = threading.Lock()
_io_pool: Optional[ThreadPoolExecutor] = None
_io_futures: Dict[Tuple[int, int], Any] = {}


def _stream(device) -> Optional["torch.cuda.Stream"]:
    if not torch.cuda.is_available():
        return None
    dev = torch.device(device)
    if dev.type != "cuda":
        return None
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _lock:
        if idx not in _side_stream:
            _side_stream[idx] = torch.cuda.Stream(device=idx)
        return _side_stream[idx]


def _io() -> ThreadPoolExecutor:
    global _io_pool
    with _lock:
        if _io_pool is None:
            _io_pool = ThreadPoolExecutor(max_workers=2, thread_name_prefix="t1-gds")
        return _io_pool


def reset_prefetch_state() -> None:
    """Drop pending prefetches (e.g. after an aborted backward)."""
    with _lock:
        _prefetched.clear()


class SlidingCheckpoint(saved_tensors_hooks):
    def __init__(
        self,
        layer_idx: int,
        layer_tensors: Optional[List[List[torch.Tensor]]] = None,
        gds_offload: bool = False,
        file_paths: Optional[List[List[str]]] = None,
        is_last_layer: bool = False,
        no_mask: bool = False,
        device: str = "cuda:0",
        pin_memory: bool = True,
        stream: Optional["torch.cuda.Stream"] = None,
    ):
        self.layer = layer_idx - 1  # 0-based slot index
        self.device = torch.device(device)
        self.is_last_layer = is_last_layer
        self.no_mask = no_mask
        self.pin_memory = pin_memory
        self.gds = gds_offload
        self.layer_tensors = layer_tensors
        self.file_paths = file_paths
        if gds_offload and file_paths is None:
            raise ValueError("file_paths is required when gds_offload=True")
        self.stream = stream or _stream(self.device)
        self.pack_count = 0
        self.unpack_count = 0
        self._keep: List[torch.Tensor] = []
        super().__init__(self._pack, self._unpack)

    # ------------------------------------------------------------- helpers
    def _offloading(self, t: torch.Tensor) -> bool:
        return (t.is_cuda and self.stream is not None and not self.is_last_layer
                and t.numel() > 0 and (self.layer_tensors is not None or self.gds))

    def _slot(self, layer: int, k: int, like: torch.Tensor) -> torch.Tensor:
        if self.layer_tensors is not None:
            slot = self.layer_tensors[layer][k]
            if slot.numel() < like.numel():
                raise ValueError(f"layer {layer + 1} slot {k} holds {slot.numel()} elements, "
                                 f"tensor has {like.numel()}")
            return slot.view(-1)[: like.numel()].view(like.shape) if slot.dtype == like.dtype else \
                slot.view(like.dtype).view(-1)[: like.numel()].view(like.shape)
        return torch.empty(like.shape, dtype=like.dtype, pin_memory=self.pin_memory)

    # --------------------------------------------------------------- hooks
    def _pack(self, t: torch.Tensor):
        if not self._offloading(t):
            return ("keep", t)
        k = self.pack_count
        self.pack_count += 1
        slot = self._slot(self.layer, k, t)
        ready = torch.cuda.current_stream(t.device).record_event()
        self.stream.wait_event(ready)
        with torch.cuda.stream(self.stream):
            slot.copy_(t, non_blocking=True)
            t.record_stream(self.stream)
        done = self.stream.record_event()
        if self.gds:
            path = self.file_paths[self.layer][k]

            def write(slot=slot, done=done, path=path):
                done.synchronize()
                with open(path, "wb") as f:
                    f.write(memoryview(slot.contiguous().view(torch.uint8).numpy()))

            _io_futures[(self.layer, k)] = _io().submit(write)
        return ("host", k, t.device, t.shape, t.dtype, slot, done)

    def _prefetch(self, layer: int, metas: List[tuple]) -> None:
        bufs = []
        for (k, shape, dtype, slot, done) in metas:
            if self.gds:
                fut = _io_futures.pop((layer, k), None)
                if fut is not None:
                    fut.result()
                with open(self.file_paths[layer][k], "rb") as f:
                    f.readinto(memoryview(slot.view(torch.uint8).numpy()))
            self.stream.wait_event(done)
            with torch.cuda.stream(self.stream):
                # allocated on the side stream, which writes it (memory freed by
                # the compute stream may still be in use by its queued kernels)
                buf = torch.empty(shape, dtype=dtype, device=self.device)
                buf.copy_(slot, non_blocking=True)
            bufs.append(buf)
        ev = self.stream.record_event()
        with _lock:
            _prefetched[layer] = (bufs, ev)

    def _unpack(self, packed):
        if packed[0] == "keep":
            return packed[1]
        _, k, device, shape, dtype, slot, done = packed
        if self.unpack_count == 0:
            # prefetch the previous layer's slots (reuse this layer's shapes)
            prev = self.layer - 1
            if prev >= 0 and self.layer_tensors is not None:
                metas = []
                for j, s in enumerate(self.layer_tensors[prev]):
                    metas.append((j, s.shape, s.dtype, s, done))
                self._prefetch(prev, metas)
        self.unpack_count += 1
        with _lock:
            entry = _prefetched.get(self.layer)
        if entry is not None and k < len(entry[0]) and entry[0][k].shape == shape and entry[0][k].dtype == dtype:
            bufs, ev = entry
            torch.cuda.current_stream(device).wait_event(ev)
            out = bufs[k]
            if self.no_mask or self.unpack_count >= len(bufs):
                with _lock:
                    _prefetched.pop(self.layer, None)
            return out
        # not prefetched (first layer of the backward, or shapes differ)
        if self.gds:
            fut = _io_futures.pop((self.layer, k), None)
            if fut is not None:
                fut.result()
        out = torch.empty(shape, dtype=dtype, device=device)
        torch.cuda.current_stream(device).wait_event(done)
        out.copy_(slot, non_blocking=True)
        return out


def save_on_cpu(pin_memory: bool = True):
    """Plain offload of every saved tensor (torch's ``save_on_cpu``)."""
    return torch.autograd.graph.save_on_cpu(pin_memory=pin_memory)
