"""Non-Llama HF causal LMs (here Qwen2: q/k/v biases) train through the
generic layer path of the engine; compared with HF + torch.optim.AdamW."""
import os
import tempfile

import pytest
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.slide_fsdp import SlideFSDP

transformers = pytest.importorskip("transformers")


def _tiny_qwen2():
    cfg = transformers.Qwen2Config(vocab_size=256, hidden_size=64, intermediate_size=128,
                                   num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                                   max_position_embeddings=128, tie_word_embeddings=False,
                                   attn_implementation="eager")
    torch.manual_seed(0)
    m = transformers.Qwen2ForCausalLM(cfg).float()
    # non-zero biases so that their gradients are exercised
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith(".bias"):
                p.normal_(0, 0.02)
    return m


def test_generic_qwen2_matches_hf_adamw():
    model = _tiny_qwen2()
    oracle = _tiny_qwen2()
    oracle.load_state_dict(model.state_dict())
    opt = torch.optim.AdamW(oracle.parameters(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3, weight_decay=0.01))
    assert eng.generic
    g = torch.Generator().manual_seed(1)
    try:
        for _ in range(3):
            ids = torch.randint(0, 256, (2, 32), generator=g)
            ours = float(eng(input_ids=ids, labels=ids).loss)
            opt.zero_grad()
            theirs = oracle(input_ids=ids, labels=ids).loss
            theirs.backward()
            opt.step()
            assert abs(ours - float(theirs)) < 1e-5 * abs(float(theirs))
        eng.wait_for_updates()
        master = dict(eng.named_master_tensors())
        assert set(master) == {n for n, _ in oracle.named_parameters()}
        for n, p in oracle.named_parameters():
            d = (master[n].view(p.shape) - p.detach()).abs()
            assert (d > 1e-4).float().mean().item() < 1e-3, n
            assert d.max().item() < 3 * 2 * 1e-3, n
        # inference logits
        ids = torch.randint(0, 256, (1, 16), generator=g)
        out = eng(input_ids=ids).logits
        with torch.no_grad():
            for n, p in oracle.named_parameters():
                p.copy_(master[n].view(p.shape))
            expect = oracle(input_ids=ids).logits
        assert torch.allclose(out, expect, atol=1e-4)
        # HF checkpoint of the generic model reloads into HF
        with tempfile.TemporaryDirectory() as d:
            eng.save_pretrained(d)
            re = transformers.Qwen2ForCausalLM.from_pretrained(d, torch_dtype=torch.float32)
            for n, p in re.named_parameters():
                assert torch.equal(p.detach(), master[n].view(p.shape)), n
            assert os.path.exists(os.path.join(d, "config.json"))
    finally:
        eng.close()


def test_generic_meta_model_initialises():
    cfg = transformers.Qwen2Config(vocab_size=128, hidden_size=32, intermediate_size=64,
                                   num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1,
                                   tie_word_embeddings=False)
    with torch.device("meta"):
        model = transformers.Qwen2ForCausalLM(cfg)
    eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.float32, device="cpu"))
    try:
        m = dict(eng.named_master_tensors())
        assert torch.all(m["model.layers.0.self_attn.q_proj.bias"] == 0)
        assert torch.all(m["model.norm.weight"] == 1)
        ids = torch.randint(0, 128, (1, 16))
        assert torch.isfinite(eng(input_ids=ids, labels=ids).loss)
    finally:
        eng.close()


def test_train_cli_runs_a_non_llama_checkpoint(tmp_path):
    import subprocess
    import sys

    cfg = transformers.Qwen2Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=False)
    transformers.Qwen2ForCausalLM(cfg).save_pretrained(str(tmp_path / "ckpt"))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "train.py"), "--model-path", str(tmp_path / "ckpt"),
                        "--device", "cpu", "--batch-size", "2", "--seq-length", "32", "--max-steps", "2",
                        "--num-epochs", "1", "--output-dir", str(tmp_path / "out")],
                       capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "Model type: qwen2" in r.stdout and "Training completed" in r.stdout


def test_generic_exact_grad_clip_matches_hf():
    """One process: the global norm over every layer (biases included) is
    clipped before the updates, as clip_grad_norm_ + AdamW.step."""
    clip, eps = 0.05, 1e-2
    model = _tiny_qwen2()
    oracle = _tiny_qwen2()
    oracle.load_state_dict(model.state_dict())
    opt = torch.optim.AdamW(oracle.parameters(), lr=1e-3, eps=eps, weight_decay=0.01)
    eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3, weight_decay=0.01,
                                           adam_eps=eps, exact_grad_clip=True, clip_grad_norm=clip))
    g = torch.Generator().manual_seed(3)
    try:
        for _ in range(3):
            ids = torch.randint(0, 256, (2, 32), generator=g)
            eng(input_ids=ids, labels=ids)
            opt.zero_grad()
            oracle(input_ids=ids, labels=ids).loss.backward()
            norm = float(torch.nn.utils.clip_grad_norm_(oracle.parameters(), clip))
            opt.step()
            eng.wait_for_updates()
            assert norm > 10 * clip and abs(eng.last_grad_norm - norm) < 1e-4 * norm
        master = dict(eng.named_master_tensors())
        for n, p in oracle.named_parameters():
            assert (master[n].view(p.shape) - p.detach()).abs().max().item() < 1e-5, n
    finally:
        eng.close()
