"""Streams and events that degrade to synchronous no-ops on the CPU, so the
engine's schedule runs unchanged in the CPU/gloo tests."""
from __future__ import annotations

import contextlib
from typing import Optional

import torch


class Stream:
    def __init__(self, device: torch.device, priority: int = 0):
        self.device = device
        self.s = torch.cuda.Stream(device=device, priority=priority) if device.type == "cuda" else None

    def ctx(self):
        return torch.cuda.stream(self.s) if self.s is not None else contextlib.nullcontext()

    def wait(self, ev: Optional["Event"]) -> None:
        if self.s is not None and ev is not None and ev.e is not None:
            self.s.wait_event(ev.e)

    def record(self) -> "Event":
        ev = Event(self.device)
        ev.record(self)
        return ev

    def synchronize(self) -> None:
        if self.s is not None:
            self.s.synchronize()


def current_stream(device: torch.device) -> Stream:
    st = Stream.__new__(Stream)
    st.device = device
    st.s = torch.cuda.current_stream(device) if device.type == "cuda" else None
    return st


class Event:
    def __init__(self, device: torch.device, timing: bool = False):
        self.device = device
        self.e = torch.cuda.Event(enable_timing=timing) if device.type == "cuda" else None
        self.recorded = False

    def record(self, stream: Optional[Stream] = None) -> "Event":
        if self.e is not None:
            if stream is None or stream.s is None:
                self.e.record(torch.cuda.current_stream(self.device))
            else:
                self.e.record(stream.s)
        self.recorded = True
        return self

    def synchronize(self) -> None:
        if self.e is not None:
            self.e.synchronize()

    def query(self) -> bool:
        return True if self.e is None else self.e.query()

    def elapsed_ms(self, end: "Event") -> float:
        if self.e is None:
            return 0.0
        return self.e.elapsed_time(end.e)
