"""GPU multi-tensor Adam/AdamW (the reference's FusedAdam extension,
optimizer/layer_adam/csrc/fused_adam_frontend.cpp:8-25 and
multi_tensor_adam.cu, which it builds with builder.py:127-477 but never uses).

``multi_tensor_adam`` keeps the reference's entry point; ``FusedAdam`` is a
``torch.optim.Optimizer`` on top of it for GPU-resident parameters (the
engine itself keeps the optimizer on the host; this serves users who train
small parts on the GPU, e.g. the embedding of a resident model)."""
from __future__ import annotations

from typing import Iterable, List

import torch

from .. import _native

ADAM_MODE_L2 = 0
ADAM_MODE_ADAMW = 1


def multi_tensor_adam(chunk_size: int, noop_flag: torch.Tensor, tensor_lists: List[List[torch.Tensor]],
                      lr: float, beta1: float, beta2: float, epsilon: float, step: int, mode: int,
                      bias_correction: int, weight_decay: float) -> None:
    """In-place update of ``tensor_lists = [grads, params, exp_avgs,
    exp_avg_sqs]`` (one dtype per call: fp32, fp16, bf16 or fp64)."""
    _native.cuda().multi_tensor_adam(int(chunk_size), noop_flag, tensor_lists, float(lr), float(beta1),
                                     float(beta2), float(epsilon), int(step), int(mode),
                                     int(bias_correction), float(weight_decay))


class FusedAdam(torch.optim.Optimizer):
    """Adam (``adam_w_mode=False``: L2 regularisation) or AdamW on CUDA
    tensors, one kernel launch per dtype per group (per 192 tensors)."""

    def __init__(self, params: Iterable, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, adam_w_mode: bool = True, bias_correction: bool = True,
                 chunk_size: int = 65536):
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay,
                        bias_correction=bias_correction)
        super().__init__(params, defaults)
        self.mode = ADAM_MODE_ADAMW if adam_w_mode else ADAM_MODE_L2
        self.chunk_size = chunk_size
        self._noop = None

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            b1, b2 = group["betas"]
            group["step"] = group.get("step", 0) + 1
            by_dtype = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("FusedAdam does not support sparse gradients")
                st = self.state[p]
                if not st:
                    st["exp_avg"] = torch.zeros_like(p)
                    st["exp_avg_sq"] = torch.zeros_like(p)
                lists = by_dtype.setdefault(p.dtype, [[], [], [], []])
                lists[0].append(p.grad.contiguous())
                lists[1].append(p.data)
                lists[2].append(st["exp_avg"])
                lists[3].append(st["exp_avg_sq"])
            for dt, lists in by_dtype.items():
                if self._noop is None or self._noop.device != lists[1][0].device:
                    self._noop = torch.zeros(1, dtype=torch.int32, device=lists[1][0].device)
                multi_tensor_adam(self.chunk_size, self._noop, lists, group["lr"], b1, b2, group["eps"],
                                  group["step"], self.mode, 1 if group["bias_correction"] else 0,
                                  group["weight_decay"])
        return loss
