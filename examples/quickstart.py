"""Smallest use of the public API: a tiny Llama-architecture model trained
for a few steps, on the CPU (no GPU needed) or on cuda:0.

    python examples/quickstart.py [--device cuda:0] [--steps 5]

The same calls run the 8B model on a B200 (``LlamaConfig.llama31_8b()``);
``train.py`` and ``bench.py`` are the full drivers.
"""
import argparse
import os
import sys
import tempfile

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from test1_b200 import SlideFSDPConfig  # noqa: E402
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM  # noqa: E402
from test1_b200.slide_fsdp import SlideFSDP  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--steps", type=int, default=5)
    a = ap.parse_args()
    dev = torch.device(a.device)
    cfg = LlamaConfig.tiny()
    if dev.type == "cuda":  # the sm_100a attention kernels take head_dim 128
        cfg = LlamaConfig(vocab_size=4096, hidden_size=512, intermediate_size=1536, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2)
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    model = LlamaForCausalLM(cfg, device="meta")  # weights are created in host memory by the engine
    engine = SlideFSDP(model, SlideFSDPConfig(dtype=dtype, device=dev, lr=1e-3))
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=g)
    for step in range(a.steps):
        out = engine(input_ids=ids, labels=ids)  # forward + backward + host AdamW update
        print(f"step {step}: loss {float(out.loss):.4f}")
    with tempfile.TemporaryDirectory() as d:
        engine.save_pretrained(d)  # HF layout
        print("saved:", sorted(os.listdir(d)))
    engine.close()


if __name__ == "__main__":
    main()
