"""In-place fp32 <-> (bf16 plane, residual plane) relayout.

An fp32 tensor of N elements can be rearranged, in its own storage, into N
bf16 "high" halves followed by N 16-bit "low" halves.  After adding 0x8000 to
every 32-bit pattern first, the high half is the fp32 value rounded to bf16
(ties away from zero in magnitude), so the first N bf16 elements are a usable
bf16 copy with no extra memory, and the transformation is exactly invertible.
Same capability as the reference's utils/param_reuse.py:4-56.
"""
from __future__ import annotations

from typing import Iterable

import torch

_BIAS = 0x8000


def fp32_to_split_planes_(t: torch.Tensor) -> torch.Tensor:
    """fp32 tensor -> same storage holding [bf16 plane (N) | low plane (N)].
    Returns the bf16 view of the first plane."""
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError("expects a contiguous fp32 tensor")
    n = t.numel()
    i32 = t.view(torch.int32)
    i32.add_(_BIAS)
    halves = t.view(torch.int16).view(n, 2)  # little endian: [:, 0] low, [:, 1] high
    planes = torch.stack([halves[:, 1], halves[:, 0]], 0).contiguous()
    t.view(torch.int16).copy_(planes.view(-1))
    return t.view(torch.bfloat16)[:n]


def split_planes_to_fp32_(t: torch.Tensor) -> torch.Tensor:
    """Inverse of fp32_to_split_planes_."""
    n = t.numel()
    planes = t.view(torch.int16).view(2, n)
    inter = torch.stack([planes[1], planes[0]], 1).contiguous()
    t.view(torch.int16).copy_(inter.view(-1))
    t.view(torch.int32).sub_(_BIAS)
    return t


def fp32_tensors_to_bf16_tensors(tensors: Iterable[torch.Tensor]):
    return [fp32_to_split_planes_(t) for t in tensors]


def bf16_tensors_to_fp32_tensors(tensors: Iterable[torch.Tensor]):
    return [split_planes_to_fp32_(t) for t in tensors]
