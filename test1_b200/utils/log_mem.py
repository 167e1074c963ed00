"""One-line device memory report (allocated / reserved / peak) for logs
(the figures of the reference's utils/log_mem.py:5-14)."""
from __future__ import annotations

import torch


def log_memory_stats(tag: str = "", device=None) -> str:
    if not torch.cuda.is_available():
        return f"[{tag}] cuda unavailable"
    dev = device if device is not None else torch.cuda.current_device()
    gb = 1024 ** 3
    a = torch.cuda.memory_allocated(dev) / gb
    r = torch.cuda.memory_reserved(dev) / gb
    p = torch.cuda.max_memory_allocated(dev) / gb
    return f"[{tag}] allocated {a:.2f} GiB | reserved {r:.2f} GiB | peak {p:.2f} GiB"
