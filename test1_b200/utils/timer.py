"""Per-layer, per-operation timing with CUDA events (no host sync until read;
the reference's LayerTimer, utils/timer.py:4-29, stores durations its caller
measured).

    t = LayerTimer(); t.start(3, "h2d"); ...; t.stop(3, "h2d"); t.summary()
"""
from __future__ import annotations

from collections import defaultdict
from typing import Dict, List, Tuple

import torch


class LayerTimer:
    def __init__(self, enabled: bool = True):
        self.enabled = enabled and torch.cuda.is_available()
        self._open: Dict[Tuple[int, str], torch.cuda.Event] = {}
        self._pairs: Dict[Tuple[int, str], List[Tuple[torch.cuda.Event, torch.cuda.Event]]] = defaultdict(list)

    def start(self, layer: int, op: str, stream=None) -> None:
        if not self.enabled:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        self._open[(layer, op)] = e

    def stop(self, layer: int, op: str, stream=None) -> None:
        if not self.enabled:
            return
        s = self._open.pop((layer, op), None)
        if s is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        self._pairs[(layer, op)].append((s, e))

    def summary(self) -> Dict[str, Dict[str, float]]:
        """{op: {"total_ms", "count", "mean_ms"}} (synchronises)."""
        out: Dict[str, Dict[str, float]] = {}
        for (layer, op), pairs in self._pairs.items():
            for s, e in pairs:
                e.synchronize()
                d = out.setdefault(op, {"total_ms": 0.0, "count": 0})
                d["total_ms"] += s.elapsed_time(e)
                d["count"] += 1
        for d in out.values():
            d["mean_ms"] = d["total_ms"] / max(1, d["count"])
        return out

    def reset(self) -> None:
        self._open.clear()
        self._pairs.clear()
