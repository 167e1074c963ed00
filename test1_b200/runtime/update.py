"""Host-side optimizer scheduler.

One thread per rank runs LayerAdam steps.  Work items become runnable when
their gradient has reached host memory (a CUDA event).  Among runnable items
the *lowest layer index* runs first: the next forward pass consumes layers in
ascending order while the backward produces gradients in descending order, so
finishing low layers first lets the optimizer tail overlap the next forward
instead of stalling it (the reference runs updates strictly in arrival
order, layer_state.py:439-442).

Completion is published through a per-layer monotonic counter in a host
region shared by all local ranks: a rank that updated its shard of layer i
increments counter[i]; a rank about to copy layer i to its GPU waits until
counter[i] >= updaters * completed_steps.  Waits are bounded and raise
``TimeoutError`` naming the layer (a dead peer never hangs the survivors).
"""
from __future__ import annotations

import heapq
import itertools
import threading
import time
from typing import Callable, List, Optional

import torch

from .. import _native
from .device import Event


class UpdateItem:
    __slots__ = ("layer", "seq", "event", "run")

    def __init__(self, layer: int, seq: int, event: Optional[Event], run: Callable[[], None]):
        self.layer = layer
        self.seq = seq
        self.event = event
        self.run = run

    def __lt__(self, other):
        return (self.layer, self.seq) < (other.layer, other.seq)


class UpdateScheduler:
    def __init__(self, counters: torch.Tensor, name: str = "t1-update", timeout_s: float = 600.0,
                 fifo: bool = False):
        self.counters = counters
        self.fifo = fifo
        self.timeout_s = timeout_s
        self._host = _native.host()
        self._items: List[UpdateItem] = []
        self._seq = itertools.count()
        self._cv = threading.Condition()
        self._pending = 0
        self._error: Optional[BaseException] = None
        self._stop = False
        self.busy_s = 0.0
        self.blocked_s = 0.0  # time callers spent in wait_counter
        self._thread = threading.Thread(target=self._loop, name=name, daemon=True)
        self._thread.start()

    # ---------------------------------------------------------------- api
    def submit(self, layer: int, event: Optional[Event], run: Callable[[], None]) -> None:
        self.raise_if_failed()
        with self._cv:
            self._items.append(UpdateItem(layer, next(self._seq), event, run))
            self._pending += 1
            self._cv.notify()

    def counter(self, layer: int) -> int:
        return int(self._host.counter_load(self.counters, layer))

    def publish(self, layer: int) -> None:
        self._host.counter_add(self.counters, layer, 1)

    def wait_counter(self, layer: int, target: int, timeout_s: Optional[float] = None) -> None:
        """Block until counter[layer] >= target (all updaters finished)."""
        if self._host.counter_load(self.counters, layer) >= target:
            return
        timeout = self.timeout_s if timeout_s is None else timeout_s
        t0 = time.monotonic()
        deadline = t0 + timeout
        try:
            while True:
                self.raise_if_failed()
                remaining = deadline - time.monotonic()
                if remaining <= 0:
                    raise TimeoutError(
                        f"layer {layer} parameter update timed out: counter "
                        f"{self.counter(layer)} < {target} after {timeout:.1f}s (a peer rank may have died)")
                if self._host.counter_wait_geq(self.counters, layer, target, min(remaining, 0.5)):
                    return
        finally:
            self.blocked_s += time.monotonic() - t0

    def drain(self, timeout_s: Optional[float] = None) -> None:
        timeout = self.timeout_s if timeout_s is None else timeout_s
        deadline = time.monotonic() + timeout
        with self._cv:
            while self._pending and self._error is None:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError("optimizer updates did not finish in time")
                self._cv.wait(min(left, 0.5))
        self.raise_if_failed()

    def raise_if_failed(self) -> None:
        if self._error is not None:
            raise RuntimeError("host optimizer thread failed") from self._error

    def close(self) -> None:
        with self._cv:
            self._stop = True
            self._cv.notify_all()
        self._thread.join(timeout=5)

    # ------------------------------------------------------------- thread
    def _pick(self) -> Optional[UpdateItem]:
        if self.fifo:
            best = min(self._items, key=lambda it: it.seq)
            self._items.remove(best)
            return best
        ready = [it for it in self._items if it.event is None or it.event.query()]
        if ready:
            best = min(ready)
        else:
            best = min(self._items, key=lambda it: it.seq)  # finishes first (FIFO copy stream)
        self._items.remove(best)
        return best

    def _loop(self) -> None:
        torch.set_num_threads(1)
        while True:
            with self._cv:
                while not self._items and not self._stop:
                    self._cv.wait()
                if self._stop and not self._items:
                    return
                item = self._pick()
            try:
                if item.event is not None:
                    item.event.synchronize()
                t0 = time.perf_counter()
                item.run()
                self.busy_s += time.perf_counter() - t0
            except BaseException as exc:  # propagate to the main thread
                self._error = exc
            finally:
                with self._cv:
                    self._pending -= 1
                    self._cv.notify_all()
