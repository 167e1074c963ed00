"""LayerAdam: one optimizer object, stepped one layer at a time on the host.

Public API and semantics follow the reference's LayerAdam
(optimizer/layer_adam/layer_adam.py:9-442): per-layer parameter groups
(``add_layer_params``), a per-group step counter that drives bias correction,
``step(layer_idx)`` on ``p.grad``, ``step_with_grad_views(layer_idx, views)``
on externally owned gradient buffers, ``update_learning_rate``, and optional
optimizer-state offload to NVMe with one-layer-ahead prefetch.

The arithmetic runs in the native host kernel (``test1_b200._host``:
AVX-512 / AVX2 / scalar picked at run time, fixed worker pool pinned per
rank).  Differences from the reference, all deliberate:
  * bf16/fp16 gradients are consumed directly (the reference upcasts every
    gradient view to a temporary fp32 copy first, layer_adam.py:404);
  * non-contiguous tensors are rejected instead of being updated through a
    temporary copy whose result is lost (cpu_adam_impl.cpp:211-237);
  * the engine path (``add_flat_layer`` / ``step_flat``) updates one flat
    slice per layer -- the rank's shard of the shared master -- and writes
    the bf16 shadow used for the next host-to-device copy in the same pass.
"""
from __future__ import annotations

import math
import os
import threading
from collections import OrderedDict, defaultdict
from concurrent.futures import ThreadPoolExecutor
from typing import Any, DefaultDict, Dict, Iterable, Optional

import torch

from .. import _native
from ..runtime.scratch_file import ScratchFile


class _StateOffloader:
    """Moves per-layer state tensors to files and back.

    ``offload(key, t)`` writes ``t`` to the key's nameless scratch file in
    ``<dir>`` (runtime/scratch_file.py) on a background thread and drops the in-memory tensor once written;
    ``prefetch(key)`` reads it back into a fresh tensor on the same thread
    pool; ``get(key)`` waits for the pending operation and returns the
    resident tensor.  Operations on one key are ordered (each waits for the
    previous one).
    """

    def __init__(self, directory: str):
        os.makedirs(directory, exist_ok=True)
        self.dir = directory
        self.pool = ThreadPoolExecutor(max_workers=2, thread_name_prefix="t1-optoffload")
        self.pending: Dict[Any, Any] = {}
        self.meta: Dict[Any, tuple] = {}
        self.tensors: Dict[Any, Optional[torch.Tensor]] = {}
        self.files: Dict[Any, ScratchFile] = {}  # nameless: nothing outlives the process

    def _file(self, key) -> ScratchFile:
        f = self.files.get(key)
        if f is None:
            f = self.files[key] = ScratchFile(self.dir)
        return f

    def _wait(self, key) -> None:
        f = self.pending.pop(key, None)
        if f is not None:
            f.result()

    def offload(self, key, t: torch.Tensor) -> None:
        self._wait(key)
        self.meta[key] = (t.numel(), t.dtype)
        self.tensors[key] = t

        file = self._file(key)

        def job():
            raw = t.view(torch.uint8) if t.dtype != torch.uint8 else t
            file.write(memoryview(raw.numpy()))
            self.tensors[key] = None

        self.pending[key] = self.pool.submit(job)

    def prefetch(self, key) -> None:
        self._wait(key)
        if self.tensors.get(key) is not None:
            return

        def job():
            numel, dtype = self.meta[key]
            t = torch.empty(numel, dtype=dtype)
            self.files[key].read_into(memoryview(t.view(torch.uint8).numpy()))
            self.tensors[key] = t

        self.pending[key] = self.pool.submit(job)

    def get(self, key) -> torch.Tensor:
        self._wait(key)
        t = self.tensors.get(key)
        if t is None:
            self.prefetch(key)
            self._wait(key)
            t = self.tensors[key]
        return t

    def close(self):
        self.pool.shutdown(wait=True)
        for f in self.files.values():
            f.close()
        self.files.clear()


class LayerAdam:
    """Layer-wise Adam/AdamW whose state lives in host memory."""

    def __init__(
        self,
        lr: float = 1e-3,
        bias_correction: bool = True,
        betas=(0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.0,
        adamw_mode: bool = True,
        fp32_optimizer_state: bool = True,
        num_layer: int = 0,
        nvme_offload_fraction: float = 0.0,
        offload_dir: str = "/tmp/opt_offload",
        prefetch: bool = True,
        state_dtype: Optional[torch.dtype] = None,
    ):
        if not 0.0 <= nvme_offload_fraction <= 1.0:
            raise ValueError("nvme_offload_fraction must be in [0, 1]")
        self.defaults = dict(
            lr=lr,
            bias_correction=bias_correction,
            betas=tuple(betas),
            eps=eps,
            weight_decay=weight_decay,
            adamw_mode=adamw_mode,
        )
        self.param_groups: list = []
        self._groups: Dict[int, dict] = {}
        self.fp32_optimizer_state = fp32_optimizer_state
        # explicit m/v dtype of flat layers (overrides fp32_optimizer_state)
        self.state_dtype = state_dtype
        self.num_layer = num_layer
        self.state: DefaultDict[torch.Tensor, Any] = defaultdict(dict)
        self.exp_avg_flat: "OrderedDict[int, torch.Tensor]" = OrderedDict()
        self.exp_avg_sq_flat: "OrderedDict[int, torch.Tensor]" = OrderedDict()
        self._flat_param: Dict[int, torch.Tensor] = {}
        self.nvme_offload_fraction = nvme_offload_fraction
        self.prefetch = prefetch
        self.offload_dir = offload_dir if nvme_offload_fraction > 0.0 else None
        self.offloader = _StateOffloader(offload_dir) if nvme_offload_fraction > 0.0 else None
        self._host = _native.host()
        self._host.create_adam(0, lr, betas[0], betas[1], eps, weight_decay, adamw_mode, False)

    # ------------------------------------------------------------ set-up
    def _new_group(self, layer_idx: int, params: list) -> dict:
        group = {"params": params, "layer_idx": layer_idx, "step": 0, **self.defaults}
        if layer_idx in self._groups:
            raise ValueError(f"layer {layer_idx} already registered with LayerAdam")
        self._groups[layer_idx] = group
        self.param_groups.append(group)
        return group

    def _state_dtype(self, like: torch.dtype) -> torch.dtype:
        return torch.float32 if self.fp32_optimizer_state else like

    def add_layer_params(self, layer_idx: int, params: Iterable[torch.nn.Parameter]) -> int:
        """Register a layer's parameters (a per-layer group with flat state).
        Returns ``layer_idx``, or -1 if the layer has no parameters."""
        params = list(params)
        if not params:
            return -1
        self._new_group(layer_idx, params)
        numel = sum(p.numel() for p in params)
        sdt = self._state_dtype(params[0].dtype)
        self.exp_avg_flat[layer_idx] = torch.zeros(numel, dtype=sdt)
        self.exp_avg_sq_flat[layer_idx] = torch.zeros(numel, dtype=sdt)
        off = 0
        for p in params:
            n = p.numel()
            self.state[p]["exp_avg"] = self.exp_avg_flat[layer_idx][off:off + n].view(p.shape)
            self.state[p]["exp_avg_sq"] = self.exp_avg_sq_flat[layer_idx][off:off + n].view(p.shape)
            off += n
        self._after_register(layer_idx)
        return layer_idx

    def add_flat_layer(self, layer_idx: int, flat_param) -> int:
        """Register one contiguous 1-D parameter slice (the engine path: the
        rank's shard of the layer's shared fp32 master).  ``flat_param`` is an
        fp32 tensor, or a (hi, lo) pair of 16-bit planes holding the fp32
        values split (see csrc/host/host_kernels.h, kSplit)."""
        planes = isinstance(flat_param, (tuple, list))
        ts = list(flat_param) if planes else [flat_param]
        for t in ts:
            if t.dim() != 1 or not t.is_contiguous():
                raise ValueError("flat_param must be contiguous 1-D tensor(s)")
        if planes and (len(ts) != 2 or ts[0].numel() != ts[1].numel()):
            raise ValueError("split master needs two planes of equal size")
        self._new_group(layer_idx, [])
        n = ts[0].numel()
        if self.state_dtype is not None:
            sdt = self.state_dtype
        else:
            sdt = torch.float32 if (planes or self.fp32_optimizer_state) else ts[0].dtype
        self.exp_avg_flat[layer_idx] = torch.zeros(n, dtype=sdt)
        self.exp_avg_sq_flat[layer_idx] = torch.zeros(n, dtype=sdt)
        self._flat_param[layer_idx] = tuple(ts) if planes else flat_param
        self._after_register(layer_idx)
        return layer_idx

    def _after_register(self, layer_idx: int) -> None:
        if self.offloader is not None and layer_idx != self.num_layer - 1:
            self._offload_layer(layer_idx)

    # ---------------------------------------------------- NVMe state offload
    def _offloaded_names(self):
        return ["exp_avg", "exp_avg_sq"] if self.nvme_offload_fraction > 0.5 else ["exp_avg"]

    def _flat_dict(self, name):
        return self.exp_avg_flat if name == "exp_avg" else self.exp_avg_sq_flat

    def _offload_layer(self, layer_idx: int) -> None:
        if self.offloader is None or layer_idx not in self.exp_avg_flat:
            return
        for name in self._offloaded_names():
            flat = self._flat_dict(name)
            t = flat[layer_idx]
            if t is None:
                continue
            self.offloader.offload((layer_idx, name), t)
            flat[layer_idx] = None
            for p in self._groups[layer_idx]["params"]:
                self.state[p].pop(name, None)

    def _load_layer(self, layer_idx: int) -> None:
        if self.offloader is None:
            return
        if layer_idx < 0:
            layer_idx += self.num_layer
        if layer_idx not in self.exp_avg_flat:
            return
        for name in self._offloaded_names():
            if self._flat_dict(name)[layer_idx] is None:
                self.offloader.prefetch((layer_idx, name))

    def _ensure_resident(self, layer_idx: int) -> None:
        if self.offloader is None:
            return
        for name in self._offloaded_names():
            flat = self._flat_dict(name)
            if flat[layer_idx] is None:
                flat[layer_idx] = self.offloader.get((layer_idx, name))
                off = 0
                for p in self._groups[layer_idx]["params"]:
                    n = p.numel()
                    self.state[p][name] = flat[layer_idx][off:off + n].view(p.shape)
                    off += n

    def _pre_step(self, layer_idx: int) -> None:
        if self.offloader is None:
            return
        self._ensure_resident(layer_idx)
        if self.prefetch:
            self._load_layer(layer_idx - 1)

    def _post_step(self, layer_idx: int) -> None:
        if self.offloader is None:
            return
        self._offload_layer(layer_idx)

    # --------------------------------------------------------------- steps
    def _group(self, layer_idx: int) -> dict:
        try:
            return self._groups[layer_idx]
        except KeyError:
            raise KeyError(f"layer {layer_idx} was never registered with LayerAdam") from None

    def _kernel(self, group: dict, p: torch.Tensor, g: Optional[torch.Tensor], m, v,
                shadow=None, grad_scale: float = 1.0) -> None:
        beta1, beta2 = group["betas"]
        self._host.adam_step(
            p.reshape(-1), None if g is None else g.reshape(-1), m.reshape(-1), v.reshape(-1),
            None if shadow is None else shadow.reshape(-1), group["step"], group["lr"], beta1,
            beta2, group["eps"], group["weight_decay"], group["bias_correction"],
            group["adamw_mode"], grad_scale,
        )

    @torch.no_grad()
    def step(self, layer_idx: Optional[int] = None, closure=None):
        """Update one layer (or all layers when ``layer_idx`` is None) from
        ``p.grad``.  Parameters without a gradient are skipped."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if layer_idx is None:
            if self.offloader is not None:
                raise RuntimeError("with NVMe state offload, layers must be stepped one at a time")
            groups = list(self._groups.values())
        else:
            groups = [self._group(layer_idx)]
            self._pre_step(layer_idx)
        for group in groups:
            group["step"] += 1
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.device.type != "cpu":
                    raise RuntimeError(f"LayerAdam updates host tensors only, got {p.device}")
                st = self.state[p]
                self._kernel(group, p.data, p.grad.data, st["exp_avg"], st["exp_avg_sq"])
        if layer_idx is not None:
            self._post_step(layer_idx)
        return loss

    @torch.no_grad()
    def step_with_grad_views(self, layer_idx: Optional[int] = None,
                             grad_views: Optional[Dict[torch.nn.Parameter, torch.Tensor]] = None,
                             closure=None):
        """Like ``step`` but the gradient of each parameter comes from
        ``grad_views[param]`` (any float dtype, host memory)."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        groups = list(self._groups.values()) if layer_idx is None else [self._group(layer_idx)]
        if layer_idx is not None:
            self._pre_step(layer_idx)
        for group in groups:
            group["step"] += 1
            for p in group["params"]:
                g = grad_views.get(p) if grad_views else None
                if g is None:
                    continue
                if p.numel() != g.numel():
                    raise ValueError("parameter and gradient sizes differ")
                st = self.state[p]
                self._kernel(group, p.data, g, st["exp_avg"], st["exp_avg_sq"])
        if layer_idx is not None:
            self._post_step(layer_idx)
        return loss

    @torch.no_grad()
    def step_flat(self, layer_idx: int, grad: Optional[torch.Tensor],
                  shadow: Optional[torch.Tensor] = None, grad_scale: float = 1.0,
                  lr: Optional[float] = None) -> None:
        """Engine path: update the flat slice registered with
        ``add_flat_layer`` from ``grad`` (same numel, any float dtype; None =
        zero gradient), writing the low-precision ``shadow`` in the same
        pass.  ``lr`` overrides the group's learning rate for this update (the
        engine passes the rate that was current when the step ran)."""
        group = self._group(layer_idx)
        self._pre_step(layer_idx)
        group["step"] += 1
        if lr is not None:
            group = dict(group, lr=lr)
        param = self._flat_param[layer_idx]
        if isinstance(param, tuple):
            beta1, beta2 = group["betas"]
            self._host.adam_step_split(
                param[0], param[1], grad, self.exp_avg_flat[layer_idx], self.exp_avg_sq_flat[layer_idx],
                group["step"], group["lr"], beta1, beta2, group["eps"], group["weight_decay"],
                group["bias_correction"], group["adamw_mode"], grad_scale)
        else:
            self._kernel(group, param, grad, self.exp_avg_flat[layer_idx],
                         self.exp_avg_sq_flat[layer_idx], shadow, grad_scale)
        self._post_step(layer_idx)

    def update_learning_rate(self, new_lr: float) -> None:
        self.defaults["lr"] = new_lr
        for group in self.param_groups:
            group["lr"] = new_lr

    # ----------------------------------------------------------- state I/O
    def state_dict_for_layer(self, layer_idx: int) -> dict:
        group = self._group(layer_idx)
        self._ensure_resident(layer_idx)
        return {
            "step": group["step"],
            "exp_avg": self.exp_avg_flat[layer_idx],
            "exp_avg_sq": self.exp_avg_sq_flat[layer_idx],
        }

    def load_state_for_layer(self, layer_idx: int, state: dict) -> None:
        group = self._group(layer_idx)
        group["step"] = int(state["step"])
        self._ensure_resident(layer_idx)
        self.exp_avg_flat[layer_idx].copy_(state["exp_avg"])
        self.exp_avg_sq_flat[layer_idx].copy_(state["exp_avg_sq"])

    def close(self) -> None:
        if self.offloader is not None:
            self.offloader.close()
            self.offloader = None

    def __del__(self):
        try:
            self._host.destroy_adam(0)
        except Exception:
            pass


def reference_adamw_(p: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor, step: int,
                     lr: float, beta1: float, beta2: float, eps: float, wd: float,
                     bias_correction: bool = True, adamw: bool = True) -> None:
    """Plain-PyTorch restatement of the update (float64 when given float64
    tensors); the numerics oracle for the native kernel."""
    g = g.to(p.dtype)
    if wd > 0 and not adamw:
        g = g + wd * p
    m.mul_(beta1).add_(g, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step if bias_correction else 1.0
    bc2 = 1 - beta2 ** step if bias_correction else 1.0
    if wd > 0 and adamw:
        p.mul_(1 - lr * wd)
    denom = v.sqrt() / math.sqrt(bc2) + eps
    p.addcdiv_(m, denom, value=-lr / bc1)
