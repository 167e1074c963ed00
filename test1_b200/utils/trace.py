"""Per-phase step tracing for the sliding engine.

The reference has no tracer on its training path (utils/timer.py:4-29 and
utils/gpu_monitor.py:6-75 exist unused).  This one is built into the engine
and off by default (``SlideFSDPConfig.trace_path`` or ``T1_TRACE=<file>``):

* device phases are bracketed by CUDA events on the stream that runs them:
  ``h2d`` (parameter fetch, copy stream), ``fwd`` / ``bwd`` (layer compute),
  ``loss`` (output layer), ``grad_sync`` (gradient stream: reduce-scatter /
  D2H); each bracket is also an NVTX range, so an Nsight timeline shows the
  same names;
* host phases are wall-clock spans from the optimizer threads (``adam``) and
  the time the step loop spent blocked waiting for an update (``wait_update``);
* at the end of a traced step the events are resolved (one synchronisation,
  only when tracing is on) and one JSON line per step is appended:
  per-phase busy milliseconds summed over layers, per-layer detail, and --
  with several ranks -- the max over ranks of every phase total.
"""
from __future__ import annotations

import json
import threading
import time
from typing import Dict, List, Optional

import torch


class _NullSpan:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


class PhaseTracer:
    def __init__(self, device: torch.device, path: Optional[str], rank: int = 0, world: int = 1):
        self.device = device
        self.path = path
        self.enabled = bool(path)
        self.rank = rank
        self.world = world
        self.cuda = device.type == "cuda"
        self._dev: List[tuple] = []    # (phase, layer, start event, end event)
        self._host: List[tuple] = []   # (phase, layer, seconds)
        self._lock = threading.Lock()
        self._step_t0 = time.perf_counter()
        self.last: Optional[dict] = None  # record of the last traced step

    def start(self, path: Optional[str] = None) -> None:
        """Turn tracing on from the next phase (``path`` None: keep each
        step's record in ``last`` only, write no file)."""
        self.path = path
        self.enabled = True
        self._dev.clear()
        with self._lock:
            self._host.clear()
        self._step_t0 = time.perf_counter()

    def stop(self) -> None:
        self.enabled = False

    # ------------------------------------------------------------ device
    def begin(self, phase: str, layer: int, stream=None):
        """Start a device bracket on ``stream`` (a runtime Stream or None for
        the current stream); returns a token for ``end``."""
        if not self.enabled:
            return None
        if self.cuda:
            s = stream.s if stream is not None and stream.s is not None else torch.cuda.current_stream(self.device)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(s)
            torch.cuda.nvtx.range_push(f"{phase}[{layer}]")
            return (phase, layer, ev, s)
        return (phase, layer, time.perf_counter(), None)

    def end(self, token) -> None:
        if token is None:
            return
        phase, layer, start, s = token
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(s)
            torch.cuda.nvtx.range_pop()
            self._dev.append((phase, layer, start, ev))
        else:
            self._host.append((phase, layer, time.perf_counter() - start))

    def span(self, phase: str, layer: int, stream=None):
        if not self.enabled:
            return _NullSpan()
        tracer = self

        class _Span:
            def __enter__(self_inner):
                self_inner.tok = tracer.begin(phase, layer, stream)
                return self_inner

            def __exit__(self_inner, *exc):
                tracer.end(self_inner.tok)
                return False

        return _Span()

    # -------------------------------------------------------------- host
    def host(self, phase: str, layer: int, seconds: float) -> None:
        if self.enabled:
            with self._lock:
                self._host.append((phase, layer, seconds))

    # -------------------------------------------------------------- step
    def step_done(self, step: int, extra: Optional[dict] = None) -> Optional[dict]:
        """Resolve this step's brackets and append its JSON line."""
        if not self.enabled:
            return None
        if self.cuda:
            torch.cuda.synchronize(self.device)
        totals: Dict[str, float] = {}
        per_layer: Dict[str, Dict[int, float]] = {}
        for phase, layer, a, b in self._dev:
            ms = a.elapsed_time(b)
            totals[phase] = totals.get(phase, 0.0) + ms
            per_layer.setdefault(phase, {})[layer] = per_layer.get(phase, {}).get(layer, 0.0) + ms
        with self._lock:
            host = list(self._host)
            self._host.clear()
        for phase, layer, sec in host:
            totals[phase] = totals.get(phase, 0.0) + sec * 1e3
            per_layer.setdefault(phase, {})[layer] = per_layer.get(phase, {}).get(layer, 0.0) + sec * 1e3
        self._dev.clear()
        wall = (time.perf_counter() - self._step_t0) * 1e3
        self._step_t0 = time.perf_counter()
        rec = {"step": step, "rank": self.rank, "wall_ms": round(wall, 3),
               "phase_ms": {k: round(v, 3) for k, v in sorted(totals.items())},
               "layer_ms": {k: {str(i): round(x, 3) for i, x in sorted(v.items())} for k, v in per_layer.items()}}
        if self.world > 1 and torch.distributed.is_initialized():
            names = sorted(totals)
            t = torch.tensor([totals[n] for n in names] + [wall], dtype=torch.float64,
                             device=self.device if self.cuda else "cpu")
            gathered = [None] * self.world
            torch.distributed.all_gather_object(gathered, names)
            if all(g == names for g in gathered):
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                rec["max_over_ranks_ms"] = {n: round(float(x), 3) for n, x in zip(names + ["wall"], t.tolist())}
        if extra:
            rec.update(extra)
        self.last = rec
        if self.path:
            with open(self.path, "a") as f:
                f.write(json.dumps(rec) + "\n")
        return rec
