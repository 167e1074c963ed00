"""Activation checkpoint placement on the GPU path: device / pinned host /
NVMe files give bit-identical training; the NVMe mode's host-to-device copy
runs from the I/O thread."""
import pytest
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP

pytestmark = pytest.mark.gpu


def _losses(mode, tmp_path):
    # the attention kernel runs head_dim 128
    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1536, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, rope_theta=500000.0)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg, device="meta")
    eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.bfloat16, device="cuda:0", lr=1e-3, seed=3,
                                           ac_offload_mode=mode, ac_offload_dir=str(tmp_path / "a")))
    g = torch.Generator().manual_seed(4)
    out = []
    try:
        for _ in range(3):
            ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=g).cuda()
            out.append(float(eng(input_ids=ids, labels=ids).loss))
        eng.wait_for_updates()
    finally:
        eng.close()
    return out


def test_offload_modes_identical_on_gpu(tmp_path):
    base = _losses("none", tmp_path)
    assert _losses("cpu", tmp_path) == base
    assert _losses("nvme", tmp_path) == base
