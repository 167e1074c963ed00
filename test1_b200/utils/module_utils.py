"""Readable module tree with parameter counts (the reference's recursive
printer, utils/module_utils.py:3-30, shows each module's device and dtype)."""
from __future__ import annotations

import torch.nn as nn


def module_tree(module: nn.Module, name: str = "", depth: int = 0, max_depth: int = 4) -> str:
    n = sum(p.numel() for p in module.parameters(recurse=True))
    lines = [f"{'  ' * depth}{name or type(module).__name__} ({type(module).__name__}): {n:,} params"]
    if depth < max_depth:
        for child_name, child in module.named_children():
            lines.append(module_tree(child, child_name, depth + 1, max_depth))
    return "\n".join(lines)


def print_module_tree(module: nn.Module, max_depth: int = 4) -> None:
    print(module_tree(module, max_depth=max_depth))
