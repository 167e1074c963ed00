"""Checkpointed decoder-layer inputs and where they live between the
forward and the backward pass.

The engine checkpoints exactly one tensor per decoder layer: the layer's
input hidden states ``[T, hidden]`` (the reference packs the same tensor, plus
the attention mask, through ``SlidingCheckpoint``'s saved-tensor hooks,
sliding_checkpoint.py:51-131).  Modes:

  gpu   keep it in device memory (also what ``ac_offload_mode="none"`` means:
        the reference asserts in that mode, sliding_checkpoint.py:39-40)
  cpu   copy it to a page-locked host slot (one per layer) on a side stream
        during the forward; in the backward, copy layer i-1's input back
        while layer i runs (one layer ahead)
  nvme  hold no per-layer host copy: the side-stream copy lands in one of a
        small ring of page-locked staging buffers, an I/O thread writes it to
        a nameless file in ``ac_offload_dir`` (runtime/scratch_file.py: no
        file outlives the process) and frees the buffer; in the
        backward the I/O thread reads the file one layer ahead into a staging
        buffer and issues the host-to-device copy itself, so neither the
        read nor the copy sits on the compute path.  (The reference's
        GPUDirect-Storage path needs kvikio, which is absent, and its nvme
        mode asserts at start, sliding_checkpoint.py:33-36.)

The last decoder layer's input always stays on the GPU (its backward starts
right after the forward ends, as in the reference).  On a CPU-only run the
cpu and nvme modes still run (plain copies), which is how the tests cover
them without a GPU.
"""
from __future__ import annotations

import os
import queue
import threading
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Dict, Optional

import torch

from .device import Event, Stream
from .scratch_file import ScratchFile


class _StagingRing:
    """A few page-locked buffers reused for file I/O (nvme mode).  Buffers
    of an outdated size (the activation shape changed) are dropped when they
    come back."""

    def __init__(self, n: int, pin: bool):
        self.n = n
        self.pin = pin
        self.free: "queue.Queue[torch.Tensor]" = queue.Queue()
        self.nbytes = 0
        self._lock = threading.Lock()

    def acquire(self, nbytes: int) -> torch.Tensor:
        with self._lock:
            if nbytes > self.nbytes:
                self.nbytes = nbytes
                for _ in range(self.n):
                    self.free.put(torch.empty(nbytes, dtype=torch.uint8, pin_memory=self.pin))
        while True:
            buf = self.free.get()
            if buf.numel() >= nbytes and buf.numel() == self.nbytes:
                return buf

    def release(self, buf: torch.Tensor) -> None:
        if buf.numel() == self.nbytes:
            self.free.put(buf)


class ActivationStore:
    def __init__(self, mode: str, device: torch.device, d2h: Stream, h2d: Stream,
                 directory: str = "/tmp/ac_offload", staging_buffers: int = 3):
        if mode == "none":
            mode = "gpu"
        self.mode = mode
        self.device = device
        self.cuda = device.type == "cuda"
        self.d2h = d2h
        self.h2d = h2d
        self.dir = directory
        self._gpu: Dict[int, torch.Tensor] = {}
        self._host: Dict[int, torch.Tensor] = {}
        self._saved_ev: Dict[int, Event] = {}
        self._loaded_ev: Dict[int, Event] = {}
        self._write_futs: Dict[int, Future] = {}
        self._read_futs: Dict[int, Future] = {}
        self._meta: Dict[int, tuple] = {}
        self._files: Dict[int, ScratchFile] = {}  # nvme: one nameless file per layer
        self._ring = _StagingRing(staging_buffers, self.cuda) if mode == "nvme" else None
        self._io = ThreadPoolExecutor(max_workers=2, thread_name_prefix="t1-acio") if mode == "nvme" else None
        if mode == "nvme":
            os.makedirs(directory, exist_ok=True)
        self.bytes_d2h = 0
        self.bytes_h2d = 0
        self.bytes_file = 0

    # ---------------------------------------------------------------- helpers
    def _slot(self, i: int, like: torch.Tensor) -> torch.Tensor:
        t = self._host.get(i)
        if t is None or t.shape != like.shape or t.dtype != like.dtype:
            t = torch.empty(like.shape, dtype=like.dtype, pin_memory=self.cuda)
            self._host[i] = t
        return t

    def _file(self, i: int) -> ScratchFile:
        f = self._files.get(i)
        if f is None:
            f = self._files[i] = ScratchFile(self.dir)
        return f

    def _d2h_copy(self, dst: torch.Tensor, h: torch.Tensor) -> Event:
        ready = Event(self.device).record()  # h produced on the current stream
        self.d2h.wait(ready)
        with self.d2h.ctx():
            dst.copy_(h, non_blocking=True)
            if self.cuda:
                h.record_stream(self.d2h.s)
        self.bytes_d2h += h.numel() * h.element_size()
        return self.d2h.record()

    # ------------------------------------------------------------------- API
    def save(self, i: int, h: torch.Tensor, keep_on_gpu: bool = False) -> None:
        if self.mode == "gpu" or keep_on_gpu:
            self._gpu[i] = h
            return
        if self.mode == "cpu":
            self._saved_ev[i] = self._d2h_copy(self._slot(i, h), h)
            return
        # nvme: stage, write, free the staging buffer
        nbytes = h.numel() * h.element_size()
        buf = self._ring.acquire(nbytes)
        view = buf[:nbytes].view(h.dtype).view(h.shape)
        ev = self._d2h_copy(view, h)
        self._meta[i] = (h.shape, h.dtype, nbytes)
        prev = self._write_futs.pop(i, None)
        if prev is not None:
            prev.result()

        file = self._file(i)

        def write(buf=buf, ev=ev, nbytes=nbytes, file=file):
            try:
                ev.synchronize()
                file.write(memoryview(buf[:nbytes].numpy()))
            finally:
                self._ring.release(buf)

        self._write_futs[i] = self._io.submit(write)
        self.bytes_file += nbytes

    def prefetch(self, i: int) -> None:
        """Start bringing layer i's checkpoint back (call one layer ahead)."""
        if i in self._gpu or i in self._loaded_ev or i in self._read_futs:
            return
        if self.mode == "cpu":
            if i not in self._host:
                return
            slot = self._host[i]
            self.h2d.wait(self._saved_ev.get(i))
            with self.h2d.ctx():
                # allocated on the copy stream: the caching allocator then only
                # hands out memory whose previous users on that stream are done
                # (memory freed by the compute stream may still be in use by its
                # queued kernels)
                buf = torch.empty(slot.shape, dtype=slot.dtype, device=self.device)
                buf.copy_(slot, non_blocking=True)
            self._gpu[i] = buf
            self._loaded_ev[i] = self.h2d.record()
            self.bytes_h2d += buf.numel() * buf.element_size()
            return
        if self.mode != "nvme" or i not in self._meta:
            return
        shape, dtype, nbytes = self._meta[i]
        with self.h2d.ctx():  # owned by the copy stream (see the cpu mode above)
            out = torch.empty(shape, dtype=dtype, device=self.device)
        wfut = self._write_futs.pop(i, None)

        def read(i=i, out=out, nbytes=nbytes, wfut=wfut):
            if wfut is not None:
                wfut.result()
            buf = self._ring.acquire(nbytes)
            try:
                self._files[i].read_into(memoryview(buf[:nbytes].numpy()))
                src = buf[:nbytes].view(out.dtype).view(out.shape)
                if self.cuda:
                    with torch.cuda.device(self.device):
                        with self.h2d.ctx():
                            out.copy_(src, non_blocking=True)
                        ev = self.h2d.record()
                    ev.synchronize()  # the staging buffer is reused after this
                else:
                    out.copy_(src)
                    ev = None
            finally:
                self._ring.release(buf)
            return ev

        self._gpu[i] = out
        self._read_futs[i] = self._io.submit(read)
        self.bytes_h2d += nbytes

    def get(self, i: int) -> torch.Tensor:
        if i not in self._gpu:
            self.prefetch(i)
        fut = self._read_futs.pop(i, None)
        if fut is not None:
            fut.result()  # the copy into the device tensor has completed
        ev = self._loaded_ev.pop(i, None)
        if ev is not None and ev.e is not None:
            torch.cuda.current_stream(self.device).wait_event(ev.e)
        t = self._gpu.pop(i)
        if self.cuda and (ev is not None or fut is not None):
            # allocated on the copy stream, used from here on by this stream
            t.record_stream(torch.cuda.current_stream(self.device))
        return t

    def clear(self) -> None:
        for fut in self._read_futs.values():
            fut.result()
        self._read_futs.clear()
        self._gpu.clear()
        self._loaded_ev.clear()

    def close(self) -> None:
        if self._io is not None:
            for fut in list(self._write_futs.values()) + list(self._read_futs.values()):
                try:
                    fut.result()
                except Exception:
                    pass
            self._io.shutdown(wait=True)
        for f in self._files.values():
            f.close()
        self._files.clear()
        self._host.clear()
        self._gpu.clear()
