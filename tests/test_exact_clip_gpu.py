"""exact_grad_clip on the GPU path: the norm measured from the host
gradients before the updates equals the one clip_grad_norm_() reads back
from the same held gradients, and training stays finite."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_exact_grad_clip_on_cuda(cuda_device):
    from test1_b200 import SlideFSDPConfig
    from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
    from test1_b200.slide_fsdp import SlideFSDP

    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1536, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2)
    eng = SlideFSDP(LlamaForCausalLM(cfg, device="meta"),
                    SlideFSDPConfig(dtype=torch.bfloat16, device=cuda_device, lr=1e-4,
                                    exact_grad_clip=True, clip_grad_norm=0.01))
    try:
        g = torch.Generator().manual_seed(0)
        for _ in range(3):
            ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=g)
            loss = float(eng(input_ids=ids, labels=ids).loss)
            assert loss == loss and loss < 20
            eng.wait_for_updates()
            measured = eng.last_grad_norm
            assert measured is not None and measured > 0.01
            held = float(eng.clip_grad_norm_(1e30))  # reads the same host gradients, scales nothing
            assert abs(held - measured) < 1e-3 * measured, (held, measured)
    finally:
        eng.close()
