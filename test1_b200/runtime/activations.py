"""Checkpointed decoder-layer inputs and where they live between the
forward and the backward pass.

The engine checkpoints exactly one tensor per decoder layer: the layer's
input hidden states ``[T, hidden]`` (the reference packs the same tensor, plus
the attention mask, through ``SlidingCheckpoint``'s saved-tensor hooks,
sliding_checkpoint.py:51-131).  Modes:

  gpu   keep it in device memory (also what ``ac_offload_mode="none"`` means:
        the reference asserts in that mode, sliding_checkpoint.py:39-40)
  cpu   copy it to a page-locked host slot on a side stream during the
        forward; in the backward, copy layer i-1's input back while layer i
        runs (one layer ahead)
  nvme  as cpu, then a background thread writes the slot to a file under
        ``ac_offload_dir`` and reads it back one layer ahead of use (the
        reference's GPUDirect-Storage path needs kvikio, which is absent)

The last decoder layer's input always stays on the GPU (its backward starts
right after the forward ends, as in the reference).
"""
from __future__ import annotations

import os
import threading
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Dict, List, Optional

import torch

from .device import Event, Stream


class ActivationStore:
    def __init__(self, mode: str, device: torch.device, d2h: Stream, h2d: Stream,
                 directory: str = "/tmp/ac_offload"):
        if mode == "none":
            mode = "gpu"
        if device.type != "cuda" and mode != "gpu":
            mode = "gpu"  # CPU runs: nothing to offload to
        self.mode = mode
        self.device = device
        self.d2h = d2h
        self.h2d = h2d
        self.dir = directory
        self._gpu: Dict[int, torch.Tensor] = {}
        self._host: Dict[int, torch.Tensor] = {}
        self._saved_ev: Dict[int, Event] = {}
        self._loaded_ev: Dict[int, Event] = {}
        self._file_futs: Dict[int, Future] = {}
        self._io = ThreadPoolExecutor(max_workers=2, thread_name_prefix="t1-acio") if mode == "nvme" else None
        if mode == "nvme":
            os.makedirs(directory, exist_ok=True)
        self.bytes_d2h = 0
        self.bytes_h2d = 0

    def _slot(self, i: int, like: torch.Tensor) -> torch.Tensor:
        t = self._host.get(i)
        if t is None or t.shape != like.shape or t.dtype != like.dtype:
            t = torch.empty(like.shape, dtype=like.dtype, pin_memory=True)
            self._host[i] = t
        return t

    def _path(self, i: int) -> str:
        return os.path.join(self.dir, f"act-{os.getpid()}-{i}.bin")

    def save(self, i: int, h: torch.Tensor, keep_on_gpu: bool = False) -> None:
        if self.mode == "gpu" or keep_on_gpu:
            self._gpu[i] = h
            return
        ready = Event(self.device).record()  # h produced on the current stream
        slot = self._slot(i, h)
        self.d2h.wait(ready)
        with self.d2h.ctx():
            slot.copy_(h, non_blocking=True)
            h.record_stream(self.d2h.s)
        self._saved_ev[i] = self.d2h.record()
        self.bytes_d2h += h.numel() * h.element_size()
        if self.mode == "nvme":
            ev = self._saved_ev[i]

            def write(i=i, slot=slot, ev=ev):
                ev.synchronize()
                with open(self._path(i), "wb") as f:
                    f.write(memoryview(slot.view(torch.uint8).numpy()))

            self._file_futs[i] = self._io.submit(write)

    def prefetch(self, i: int) -> None:
        """Start bringing layer i's checkpoint back (call one layer ahead)."""
        if i in self._gpu or i in self._loaded_ev or i not in self._host:
            return
        slot = self._host[i]
        if self.mode == "nvme":
            fut = self._file_futs.pop(i, None)
            if fut is not None:
                fut.result()

            with open(self._path(i), "rb") as f:
                f.readinto(memoryview(slot.view(torch.uint8).numpy()))
        else:
            self.h2d.wait(self._saved_ev.get(i))
        buf = torch.empty(slot.shape, dtype=slot.dtype, device=self.device)
        with self.h2d.ctx():
            buf.copy_(slot, non_blocking=True)
        self._gpu[i] = buf
        self._loaded_ev[i] = self.h2d.record()
        self.bytes_h2d += buf.numel() * buf.element_size()

    def get(self, i: int) -> torch.Tensor:
        if i not in self._gpu:
            self.prefetch(i)
        ev = self._loaded_ev.pop(i, None)
        if ev is not None and ev.e is not None:
            torch.cuda.current_stream(self.device).wait_event(ev.e)
            self._gpu[i].record_stream(torch.cuda.current_stream(self.device))
        return self._gpu.pop(i)

    def clear(self) -> None:
        self._gpu.clear()
        self._loaded_ev.clear()

    def close(self) -> None:
        if self._io is not None:
            self._io.shutdown(wait=True)
            for i in list(self._host):
                try:
                    os.remove(self._path(i))
                except OSError:
                    pass
        self._host.clear()
        self._gpu.clear()
