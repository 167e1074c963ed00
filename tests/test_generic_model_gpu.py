"""A non-Llama HF model (Qwen2, biases) trains on the GPU through the
generic layer path: bf16 compute, host master, sliding pool."""
import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")


def test_generic_qwen2_trains_on_gpu():
    from test1_b200 import SlideFSDPConfig
    from test1_b200.slide_fsdp import SlideFSDP

    cfg = transformers.Qwen2Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=False,
                                   attn_implementation="sdpa")
    torch.manual_seed(0)
    model = transformers.Qwen2ForCausalLM(cfg).float()
    eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.bfloat16, device="cuda:0", lr=1e-3))
    assert eng.generic
    g = torch.Generator().manual_seed(1)
    losses = []
    try:
        ids = torch.randint(0, 512, (2, 64), generator=g).cuda()
        for _ in range(4):
            losses.append(float(eng(input_ids=ids, labels=ids).loss))
        eng.wait_for_updates()
    finally:
        eng.close()
    assert all(l == l and 0 < l < 20 for l in losses)
    assert losses[-1] < losses[0]  # the same batch four times: the loss goes down
