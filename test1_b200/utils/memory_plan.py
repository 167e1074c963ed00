"""Memory plan of a run before anything is allocated: host bytes on the node
(shared master, optimizer state and gradient shards of all local ranks,
cpu_reduce slots, activation checkpoints) and device bytes per GPU (the
layer pool).  The reference prints a CPU-memory estimate in its model banner
(slide_fsdp.py:683-703); this computes the engine's actual layout from the
model config and the run configuration, so a 70B run can be sized before it
starts (``train.py --plan``).

    from test1_b200.utils.memory_plan import plan_memory
    plan_memory(LlamaConfig.llama_70b(), SlideFSDPConfig(param_transfer_mode="shard"), world=8,
                batch=1, seq=2048)
"""
from __future__ import annotations

from typing import Dict

import torch

GB = 1e9


def _layer_sizes(cfg) -> Dict[str, int]:
    H, V = cfg.hidden_size, cfg.vocab_size
    return {"embed": V * H, "decoder": cfg.decoder_layer_params(), "output": V * H + H,
            "layers": cfg.num_hidden_layers}


def plan_memory(model_cfg, config, world: int = 1, batch: int = 4, seq: int = 1024) -> Dict[str, float]:
    """Bytes (as GB) the engine will hold, summed over the node's ranks for
    host memory and per GPU for device memory."""
    sz = _layer_sizes(model_cfg)
    L = sz["layers"]
    total = sz["embed"] + L * sz["decoder"] + sz["output"]
    es = torch.tensor([], dtype=config.dtype).element_size()
    if config.dtype == torch.bfloat16 and config.master_layout == "bf16":
        master = 2 * total
    elif config.dtype == torch.bfloat16 and config.master_layout == "split":
        master = 4 * total
    else:
        master = 4 * total + (2 * total if config.dtype != torch.float32 else 0)
    state_b = 2 if config.optimizer_state_dtype == "bf16" else 4
    optimizer = 2 * state_b * total  # m and v, split over the ranks but all on this node
    grads = es * total
    biggest = max(sz["embed"], sz["decoder"], sz["output"])
    slots = 0
    if world > 1 and config.grad_sync_mode == "cpu_reduce":
        cap = -(-biggest // 4096) * 4096
        slots = 4 * world * cap * es
    acts = 0
    if config.enable_activation_checkpoint and config.ac_offload_mode == "cpu":
        acts = world * (L - 1) * batch * seq * model_cfg.hidden_size * es
    host = master + optimizer + grads + slots + acts
    # device pool: pool units for decoder layers and one unit shared by the
    # embedding and the output layer, each holding parameters and gradients
    pad = lambda n: world * -(-n // world)  # shards padded to N equal parts
    dec_unit = pad(sz["decoder"]) if world > 1 else sz["decoder"]
    big_unit = pad(max(sz["embed"], sz["output"])) if world > 1 else max(sz["embed"], sz["output"])
    device_pool = (config.gpu_buffer_pool_size * dec_unit + big_unit) * 2 * es
    return {"params": float(total), "host_master_gb": master / GB, "host_optimizer_gb": optimizer / GB,
            "host_grads_gb": grads / GB, "host_cpu_reduce_slots_gb": slots / GB,
            "host_activation_offload_gb": acts / GB, "host_total_gb": host / GB,
            "device_pool_gb_per_gpu": device_pool / GB}
