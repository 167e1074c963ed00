"""SlideFSDPConfig: every knob of the layer-sliding trainer.

Same field names, defaults, accepted values and validation messages as the
reference's configuration dataclass (config.py:17-165 in LaiHOLA/Test1), so
JSON configs written for the reference load unchanged.  Fields that the
reference accepts but ignores are honoured here: ``prefetch_layers`` (units
loaded ahead), ``max_workers`` and ``clip_grad_norm`` (applied before the
updates when ``exact_grad_clip`` is set; otherwise ``clip_grad_norm_()``
reports the norm after the fact, as in the reference).

Extra fields (all optional, reference configs never set them):
    optimizer_sharding: "rank" (each rank updates 1/N of every layer, the
        default) or "rank0" (the reference's single-optimizer placement).
    fused_comm: use the fused NVLink kernels for shard all-gather and
        gpu_reduce reduce-scatter when available (else NCCL).
    shard_source: what shard mode reads from host memory: the bf16
        "shadow" (default; the high plane of the split master), moved by the
        copy engine one layer ahead and then broadcast over NVLink, 2 B per
        parameter over PCIe; or the fp32 "master", read by the gather
        kernels themselves and rounded to bf16 on the GPU, 4 B per parameter.
    shard_gather_ctas: CTAs of the NVLink broadcast kernel that runs next to
        the compute kernels in staged shard mode.
    lm_head_chunk_tokens: the output layer computes lm_head + cross-entropy
        and their gradients in chunks of this many tokens (only a
        [chunk, vocab] logits buffer exists); 0 keeps the full logits.
    host_threads: size of the per-rank host worker pool (0 = all CPUs in the
        affinity mask).
    master_layout: how the fp32 master is stored in host memory: "split"
        keeps each value as a bf16 high plane plus a 16-bit low plane (bit
        exact; the high plane doubles as the bf16 copy the GPUs load, so the
        optimizer writes no separate shadow: 2 fewer bytes of host memory
        traffic per parameter and step), "fp32" keeps plain fp32 plus a bf16
        shadow.  Only bf16 training uses "split".  "bf16" keeps bf16 weights
        only (each update rounded to nearest even), the reference's
        bf16-parameter LayerAdam mode for models whose fp32 master does not
        fit in host RAM.
    optimizer_state_dtype: dtype of LayerAdam's m and v in host memory
        ("fp32", or "bf16" to halve the state of very large models).
    exact_grad_clip: with clip_grad_norm > 0, every step scales its
        gradients so that their global L2 norm (over all layers and ranks)
        is at most clip_grad_norm before any layer is updated, as
        torch.nn.utils.clip_grad_norm_ before optimizer.step() does.  The
        updates then start after the whole backward instead of overlapping
        it.  Off by default (the reference never clips).
    host_wait_timeout_s: bound on every host-side wait for another rank
        (optimizer publication, cpu_reduce slots); expiry raises TimeoutError.
    trace_path: append one JSON line per training step with per-phase
        device times (h2d, fwd, bwd, loss, grad_sync) and host optimizer
        spans (utils/trace.py); each rank writes ``<path>.rank<r>`` when
        there are several.
    use_native_kernels: run the model on the sm_100a kernels (True) or on
        plain PyTorch ops (False; the CPU test path).
    fuse_gather_qkv: in shard mode the forward gathers each decoder layer
        inside its QKV GEMM kernel (True, default).  False gathers it with
        the standalone fused gather on the copy stream one layer ahead (as
        the backward always does), taking the gather off the forward's
        critical path at the cost of the fusion.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, fields
from typing import Optional, Tuple

import torch


@dataclass
class SlideFSDPConfig:
    # Basic configuration
    dtype: torch.dtype = torch.bfloat16
    device: Optional[torch.device] = None  # auto-detect from LOCAL_RANK

    # Parameter transfer strategy: "full" | "shard"
    param_transfer_mode: str = "full"

    # Gradient synchronization strategy: "gpu_reduce" | "cpu_reduce"
    grad_sync_mode: str = "gpu_reduce"

    # Optimizer configuration
    lr: float = 1e-5
    weight_decay: float = 0.01
    adam_betas: Tuple[float, float] = (0.9, 0.999)
    adam_eps: float = 1e-8
    bias_correction: bool = True

    # Runtime configuration
    prefetch_layers: int = 1
    max_workers: int = 1
    enable_activation_checkpoint: bool = True
    gpu_buffer_pool_size: int = 2

    # Model / training configuration (used by train.py)
    model_path: str = ""
    max_seq_length: int = 1024
    train_batch_size: int = 4
    num_epochs: int = 1
    log_every_n_steps: int = 1
    seed: int = 42
    use_liger_kernel: bool = True
    attention_implementation: str = "flash_attention_2"

    # Activation checkpoint offload: "cpu" | "nvme" | "none"
    ac_offload_mode: str = "cpu"
    ac_offload_dir: str = "/tmp/ac_offload"

    # NVMe offload for optimizer states (fraction of each layer's state)
    optimizer_nvme_offload_fraction: float = 0.0
    optimizer_offload_dir: str = "/tmp/opt_offload"

    # Gradient clipping (<= 0 disables)
    clip_grad_norm: float = 1.0

    # ---- fields without a reference counterpart --------------------------
    optimizer_sharding: str = "rank"
    fused_comm: bool = True
    shard_source: str = "shadow"  # shard fetch reads the bf16 "shadow" (copy engine) or the fp32 "master"
    shard_gather_ctas: int = 64
    lm_head_chunk_tokens: int = 2048
    host_threads: int = 0
    host_wait_timeout_s: float = 600.0  # bound on every host wait for a peer rank
    exact_grad_clip: bool = False  # clip to clip_grad_norm before the updates
    master_layout: str = "split"  # "split" (hi/lo 16-bit planes), "fp32" (fp32 + bf16 shadow) or "bf16"
    optimizer_state_dtype: str = "fp32"  # LayerAdam m/v in host memory: "fp32" or "bf16"
    use_native_kernels: Optional[bool] = None  # None: native iff device is CUDA
    fuse_gather_qkv: bool = True  # shard mode: gather each layer inside its QKV GEMM
    trace_path: Optional[str] = None  # per-phase step trace (JSON lines); env T1_TRACE also enables it

    def __post_init__(self):
        if self.param_transfer_mode not in ("full", "shard"):
            raise ValueError(
                f"param_transfer_mode must be 'full' or 'shard', got {self.param_transfer_mode}"
            )
        if self.grad_sync_mode not in ("gpu_reduce", "cpu_reduce"):
            raise ValueError(
                f"grad_sync_mode must be 'gpu_reduce' or 'cpu_reduce', got {self.grad_sync_mode}"
            )
        if self.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"dtype must be torch.bfloat16 or torch.float16, got {self.dtype}")
        if self.device is None:
            local_rank = int(os.environ.get("LOCAL_RANK", 0))
            self.device = torch.device("cuda", local_rank)
        elif isinstance(self.device, str):
            self.device = torch.device(self.device)
        if self.ac_offload_mode not in ("cpu", "nvme", "none"):
            raise ValueError(
                f"ac_offload_mode must be 'cpu', 'nvme', or 'none', got {self.ac_offload_mode}"
            )
        if self.optimizer_sharding not in ("rank", "rank0"):
            raise ValueError(
                f"optimizer_sharding must be 'rank' or 'rank0', got {self.optimizer_sharding}"
            )
        if self.master_layout not in ("split", "fp32", "bf16"):
            raise ValueError(f"master_layout must be 'split', 'fp32' or 'bf16', got {self.master_layout}")
        if self.optimizer_state_dtype not in ("fp32", "bf16"):
            raise ValueError(f"optimizer_state_dtype must be 'fp32' or 'bf16', got {self.optimizer_state_dtype}")
        if self.lm_head_chunk_tokens < 0:
            raise ValueError(f"lm_head_chunk_tokens must be >= 0, got {self.lm_head_chunk_tokens}")
        if self.shard_source not in ("master", "shadow"):
            raise ValueError(f"shard_source must be 'master' or 'shadow', got {self.shard_source}")
        if self.gpu_buffer_pool_size < 2:
            raise ValueError("gpu_buffer_pool_size must be >= 2 (current layer + prefetched layer)")
        if not 0.0 <= self.optimizer_nvme_offload_fraction <= 1.0:
            raise ValueError("optimizer_nvme_offload_fraction must be in [0, 1]")
        if isinstance(self.adam_betas, list):
            self.adam_betas = tuple(self.adam_betas)
        if self.use_native_kernels is None:
            self.use_native_kernels = self.device.type == "cuda"

    @classmethod
    def from_dict(cls, config_dict: dict) -> "SlideFSDPConfig":
        """Create a config from a dict (e.g. a JSON file).  Unknown keys are
        dropped, as in the reference."""
        d = dict(config_dict)
        if "dtype" in d and isinstance(d["dtype"], str):
            dtype_map = {
                "bf16": torch.bfloat16,
                "bfloat16": torch.bfloat16,
                "fp16": torch.float16,
                "float16": torch.float16,
                "fp32": torch.float32,
                "float32": torch.float32,
            }
            d["dtype"] = dtype_map.get(d["dtype"].lower(), torch.bfloat16)
        if "device" in d and isinstance(d["device"], str):
            d["device"] = torch.device(d["device"])
        if "adam_betas" in d and isinstance(d["adam_betas"], list):
            d["adam_betas"] = tuple(d["adam_betas"])
        valid = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in valid})

    def to_dict(self) -> dict:
        out = {}
        for f in fields(self):
            value = getattr(self, f.name)
            if isinstance(value, torch.dtype):
                value = str(value).replace("torch.", "")
            elif isinstance(value, torch.device):
                value = str(value)
            out[f.name] = value
        return out
