"""HF-layout checkpoint files (config.json, generation_config.json,
model[-0000k-of-0000n].safetensors + index), written tensor by tensor so a
model whose master copy lives in host shared memory is never duplicated in
full.  Matches the directory ``transformers``' ``save_pretrained`` produces,
which is what the reference's ``SlideFSDP.save_pretrained`` emits
(slide_fsdp.py:705-733)."""
from __future__ import annotations

import json
import os
from typing import Callable, Dict, Iterable, Optional, Tuple

import torch

SHARD_BYTES = 5 * 1024 ** 3


def save_hf_checkpoint(output_dir: str, config: dict, tensors, dtype: torch.dtype = torch.bfloat16,
                       shard_bytes: int = SHARD_BYTES) -> str:
    """``tensors``: mapping name -> tensor, or iterable of (name, numel-shape,
    callable returning the tensor) for lazy materialisation."""
    from safetensors.torch import save_file

    os.makedirs(output_dir, exist_ok=True)
    items = list(tensors.items()) if isinstance(tensors, dict) else list(tensors)
    # plan shards
    shards, cur, cur_bytes = [], [], 0
    for name, t in items:
        nbytes = (t.numel() if isinstance(t, torch.Tensor) else int(torch.tensor(t[0]).prod())) * \
            torch.tensor([], dtype=dtype).element_size()
        if cur and cur_bytes + nbytes > shard_bytes:
            shards.append(cur)
            cur, cur_bytes = [], 0
        cur.append((name, t))
        cur_bytes += nbytes
    if cur:
        shards.append(cur)
    n = len(shards)
    weight_map = {}
    total = 0
    for i, shard in enumerate(shards):
        fname = "model.safetensors" if n == 1 else f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        out = {}
        for name, t in shard:
            if not isinstance(t, torch.Tensor):
                t = t[1]()
            out[name] = t.detach().to("cpu").to(dtype).contiguous()
            total += out[name].numel() * out[name].element_size()
            weight_map[name] = fname
        save_file(out, os.path.join(output_dir, fname), metadata={"format": "pt"})
    if n > 1:
        with open(os.path.join(output_dir, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)
    cfg = dict(config)
    cfg["torch_dtype"] = str(dtype).replace("torch.", "")
    with open(os.path.join(output_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    gen = {"bos_token_id": cfg.get("bos_token_id"), "eos_token_id": cfg.get("eos_token_id"),
           "do_sample": False}
    with open(os.path.join(output_dir, "generation_config.json"), "w") as f:
        json.dump(gen, f, indent=2)
    return output_dir


def load_hf_checkpoint(path: str) -> Tuple[dict, Dict[str, torch.Tensor]]:
    """Returns (config dict, {name: tensor}) from an HF directory."""
    from safetensors.torch import load_file

    with open(os.path.join(path, "config.json")) as f:
        config = json.load(f)
    index = os.path.join(path, "model.safetensors.index.json")
    files = []
    if os.path.exists(index):
        with open(index) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
    else:
        files = ["model.safetensors"]
    tensors: Dict[str, torch.Tensor] = {}
    for fn in files:
        tensors.update(load_file(os.path.join(path, fn)))
    return config, tensors
