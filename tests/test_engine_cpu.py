"""SlideFSDP engine on CPU vs HF LlamaForCausalLM + torch.optim.AdamW."""
import pytest
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP


def _oracle(cfg, model, lr, wd):
    import transformers

    hf = transformers.LlamaForCausalLM(cfg.to_hf()).float()
    hf.config._attn_implementation = "eager"
    hf.load_state_dict({n: p.detach().clone() for n, p in model.named_parameters()})
    opt = torch.optim.AdamW(hf.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=wd)
    return hf, opt


@pytest.mark.parametrize("ckpt", [True, False])
def test_engine_matches_hf_adamw(ckpt):
    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg)
    hf, opt = _oracle(cfg, model, 1e-3, 0.01)
    conf = SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3, weight_decay=0.01,
                           enable_activation_checkpoint=ckpt)
    eng = SlideFSDP(model, conf)
    g = torch.Generator().manual_seed(1)
    try:
        for _ in range(4):
            ids = torch.randint(0, cfg.vocab_size, (2, 64), generator=g)
            ours = float(eng(input_ids=ids, labels=ids).loss)
            opt.zero_grad()
            theirs = hf(input_ids=ids, labels=ids).loss
            theirs.backward()
            opt.step()
            assert abs(ours - float(theirs)) < 1e-5 * abs(float(theirs))
        eng.wait_for_updates()
        master = dict(eng.named_master_tensors())
        for n, p in hf.named_parameters():
            d = (master[n].view(p.shape) - p.detach()).abs()
            # Adam normalises each update, so an element whose gradient is
            # ~0 can move by up to lr on rounding noise alone; require almost
            # all elements to agree tightly and none to be off by more than
            # the total step budget.
            assert (d > 1e-4).float().mean().item() < 1e-4, n
            assert d.max().item() < 4 * 2 * 1e-3, n
    finally:
        eng.close()


def test_inference_logits_match_hf():
    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg)
    hf, _ = _oracle(cfg, model, 1e-3, 0.0)
    eng = SlideFSDP(model, SlideFSDPConfig(dtype=torch.float32, device="cpu"))
    try:
        ids = torch.randint(0, cfg.vocab_size, (2, 32))
        out = eng(input_ids=ids)
        with torch.no_grad():
            expect = hf(input_ids=ids).logits
        assert torch.allclose(out.logits, expect, atol=1e-4)
    finally:
        eng.close()


def test_right_padding_mask_accepted_and_other_masks_rejected():
    cfg = LlamaConfig.tiny()
    eng = SlideFSDP(LlamaForCausalLM(cfg, device="meta"), SlideFSDPConfig(dtype=torch.float32, device="cpu"))
    try:
        ids = torch.randint(0, cfg.vocab_size, (2, 16))
        mask = torch.ones(2, 16, dtype=torch.bool)
        mask[0, 10:] = False
        labels = ids.clone()
        labels[0, 10:] = -100
        out = eng(input_ids=ids, attention_mask=mask, labels=labels)
        assert torch.isfinite(out.loss)
        mask[1, 0] = False  # left padding
        with pytest.raises(NotImplementedError):
            eng(input_ids=ids, attention_mask=mask, labels=labels)
    finally:
        eng.close()


def test_split_master_matches_fp32_master_bf16():
    """bf16 training with the split-plane master vs the plain fp32 master +
    shadow: same optimizer arithmetic; the bf16 copies differ only on exact
    rounding ties."""
    cfg = LlamaConfig.tiny()
    results = {}
    for layout in ("split", "fp32"):
        torch.manual_seed(0)
        eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.bfloat16, device="cpu",
                                                              lr=1e-3, master_layout=layout))
        g = torch.Generator().manual_seed(3)
        losses = []
        try:
            for _ in range(3):
                ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=g)
                losses.append(float(eng(input_ids=ids, labels=ids).loss))
            eng.wait_for_updates()
            assert eng.split_master == (layout == "split")
            results[layout] = (losses, {n: t.clone() for n, t in eng.named_master_tensors()})
        finally:
            eng.close()
    (la, ma), (lb, mb) = results["split"], results["fp32"]
    assert abs(la[0] - lb[0]) < 1e-3  # bf16 copies differ only on rounding ties
    for x, y in zip(la, lb):
        assert abs(x - y) < 2e-2
    for n in ma:
        d = (ma[n] - mb[n]).abs()
        # bf16 forward/backward amplify the tie differences slightly; Adam
        # bounds each element's drift by 2 lr per step
        assert (d > 1e-4).float().mean().item() < 0.1, n
        assert d.max().item() <= 3 * 2 * 1e-3 + 1e-5, n


def test_bf16_master_and_bf16_state_train():
    """The large-model mode (bf16 weights and bf16 Adam state in host
    memory): the stores are bf16 only and training tracks the fp32-master
    run closely over a few steps."""
    cfg = LlamaConfig.tiny()
    runs = {}
    for layout, sdt in (("bf16", "bf16"), ("split", "fp32")):
        torch.manual_seed(0)
        eng = SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.bfloat16, device="cpu", lr=1e-3,
                                                              master_layout=layout, optimizer_state_dtype=sdt))
        g = torch.Generator().manual_seed(5)
        try:
            if layout == "bf16":
                st = eng.layer_states[1]
                assert st.store.f32 is None and st.store.lo is None
                assert eng.layer_optimizer.exp_avg_flat[1].dtype == torch.bfloat16
            losses = []
            for _ in range(4):
                ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=g)
                losses.append(float(eng(input_ids=ids, labels=ids).loss))
            eng.wait_for_updates()
            runs[layout] = losses
        finally:
            eng.close()
    a, b = runs["bf16"], runs["split"]
    assert abs(a[0] - b[0]) < 1e-3
    for x, y in zip(a, b):
        assert abs(x - y) < 5e-2


def test_out_of_range_token_ids_and_labels_are_rejected():
    torch.manual_seed(0)
    eng = SlideFSDP(LlamaForCausalLM(LlamaConfig.tiny()), SlideFSDPConfig(dtype=torch.float32, device="cpu"))
    try:
        ids = torch.randint(0, 1024, (1, 16))
        bad = ids.clone()
        bad[0, 3] = 1024
        with pytest.raises(ValueError, match="input_ids"):
            eng(input_ids=bad, labels=ids)
        lab = ids.clone()
        lab[0, 5] = -7
        with pytest.raises(ValueError, match="labels"):
            eng(input_ids=ids, labels=lab)
        lab[0, 5] = -100  # the ignore index is fine
        assert torch.isfinite(eng(input_ids=ids, labels=lab).loss)
    finally:
        eng.close()


def test_configuration_larger_than_host_memory_is_refused(monkeypatch):
    from test1_b200.runtime import host_memory

    monkeypatch.setattr(host_memory, "mem_available_bytes", lambda: 1 << 20)
    with pytest.raises(MemoryError, match="do not fit on the node: host memory"):
        SlideFSDP(LlamaForCausalLM(LlamaConfig.tiny()), SlideFSDPConfig(dtype=torch.float32, device="cpu"))


def test_per_step_learning_rate_schedule_matches_adamw():
    """update_learning_rate between steps (no synchronisation): every update
    uses the rate of the step that produced its gradient."""
    import transformers

    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    ours = LlamaForCausalLM(cfg)
    hf = transformers.LlamaForCausalLM(cfg.to_hf()).float()
    hf.config._attn_implementation = "eager"
    hf.load_state_dict({n: p.detach().clone() for n, p in ours.named_parameters()})
    opt = torch.optim.AdamW(hf.parameters(), lr=1e-3, weight_decay=0.01)
    eng = SlideFSDP(ours, SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3, weight_decay=0.01))
    g = torch.Generator().manual_seed(7)
    try:
        for lr in (1e-3, 3e-3, 2e-4, 5e-3):
            ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=g)
            eng.update_learning_rate(lr)
            eng(input_ids=ids, labels=ids)
            for grp in opt.param_groups:
                grp["lr"] = lr
            opt.zero_grad()
            hf(input_ids=ids, labels=ids).loss.backward()
            opt.step()
        eng.wait_for_updates()
        master = dict(eng.named_master_tensors())
        for n, p in hf.named_parameters():
            d = (master[n].view(p.shape) - p.detach()).abs()
            assert (d > 1e-4).float().mean().item() < 1e-3, n
            assert d.max().item() < 4 * 5e-3, n
    finally:
        eng.close()


def test_fp16_on_the_native_llama_kernels_is_refused_early():
    cfg = SlideFSDPConfig(dtype=torch.float16, device="cpu", use_native_kernels=True)
    with pytest.raises(NotImplementedError, match="compute in bfloat16"):
        SlideFSDP(LlamaForCausalLM(LlamaConfig.tiny()), cfg)
