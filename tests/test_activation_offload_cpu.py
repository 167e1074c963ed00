"""Activation checkpoint placement (gpu / cpu / nvme) gives identical
training; the nvme mode keeps no per-layer host copy and removes its files."""
import os

import pytest
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP


def _run(mode, tmp_path, steps=3):
    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3,
                                                          ac_offload_mode=mode,
                                                          ac_offload_dir=str(tmp_path / "acts")))
    g = torch.Generator().manual_seed(2)
    losses = []
    try:
        for _ in range(steps):
            ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=g)
            losses.append(float(eng(input_ids=ids, labels=ids).loss))
        stats = eng.step_stats()
        host_slots = len(eng.acts._host)
        mode_used = eng.acts.mode
    finally:
        eng.close()
    return losses, stats, host_slots, mode_used


@pytest.mark.parametrize("mode", ["cpu", "nvme"])
def test_offload_modes_match_gpu_mode(mode, tmp_path):
    base, _, _, _ = _run("none", tmp_path)
    got, stats, host_slots, used = _run(mode, tmp_path)
    assert used == mode
    assert got == base  # the same computation, bit for bit
    L = LlamaConfig.tiny().num_hidden_layers
    assert stats["ac_d2h_bytes"] > 0 and stats["ac_h2d_bytes"] == stats["ac_d2h_bytes"]
    if mode == "nvme":
        assert host_slots == 0  # nothing kept per layer in host memory
        assert not os.listdir(tmp_path / "acts")  # the offload files have no names
    else:
        assert host_slots == L - 1  # the last layer's input stays on the device
