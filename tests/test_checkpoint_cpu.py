"""save_pretrained writes a directory HF transformers loads with identical
outputs; save_state/load_state resume is bit-exact."""
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP


def test_save_pretrained_loads_in_transformers(tmp_path):
    import transformers

    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3))
    try:
        ids = torch.randint(0, cfg.vocab_size, (2, 32))
        eng(input_ids=ids, labels=ids)
        eng.save_pretrained(str(tmp_path))
        # training can continue afterwards (the reference's save mutates params)
        eng(input_ids=ids, labels=ids)
        eng.wait_for_updates()
        hf = transformers.LlamaForCausalLM.from_pretrained(str(tmp_path), torch_dtype=torch.float32)
        assert hf.config.num_hidden_layers == cfg.num_hidden_layers
        assert (tmp_path / "config.json").exists() and (tmp_path / "generation_config.json").exists()
    finally:
        eng.close()


def test_save_state_resume_bit_exact(tmp_path):
    cfg = LlamaConfig.tiny()
    g = torch.Generator().manual_seed(5)
    data = [torch.randint(0, cfg.vocab_size, (2, 32), generator=g) for _ in range(4)]

    def make():
        torch.manual_seed(0)
        return SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3))

    a = make()
    for ids in data:
        a(input_ids=ids, labels=ids)
    a.wait_for_updates()
    ref = {n: t.clone() for n, t in a.named_master_tensors()}
    a.close()

    b = make()
    for ids in data[:2]:
        b(input_ids=ids, labels=ids)
    b.save_state(str(tmp_path))
    b.close()
    c = make()
    c.load_state(str(tmp_path))
    # optimizer step counters come from the saved state, data continues
    for ids in data[2:]:
        c(input_ids=ids, labels=ids)
    c.wait_for_updates()
    got = dict(c.named_master_tensors())
    c.close()
    for n, t in ref.items():
        assert torch.equal(got[n], t), n
