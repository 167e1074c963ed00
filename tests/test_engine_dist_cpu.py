"""Multi-rank engine on CPU/gloo (2 ranks) vs a single-process oracle:
HF LlamaForCausalLM whose per-step gradient is the mean of the ranks'
per-rank mean-loss gradients, stepped by torch.optim.AdamW."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests._dist_worker import batches, run_engine


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle(world, steps, clip=None, eps=1e-8):
    import transformers

    from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    ours = LlamaForCausalLM(cfg)
    hf = transformers.LlamaForCausalLM(cfg.to_hf()).float()
    hf.config._attn_implementation = "eager"
    hf.load_state_dict({n: p.detach().clone() for n, p in ours.named_parameters()})
    opt = torch.optim.AdamW(hf.parameters(), lr=1e-3, betas=(0.9, 0.999), eps=eps, weight_decay=0.01)
    losses, norms = [], []
    for step_batches in batches(cfg, world, steps):
        opt.zero_grad()
        per_rank = []
        for ids in step_batches:
            loss = hf(input_ids=ids, labels=ids).loss / world
            loss.backward()
            per_rank.append(float(loss) * world)
        if clip is not None:
            norms.append(float(torch.nn.utils.clip_grad_norm_(hf.parameters(), clip)))
        opt.step()
        losses.append(per_rank)
    if clip is not None:
        return losses, dict(hf.named_parameters()), norms
    return losses, dict(hf.named_parameters())


@pytest.mark.parametrize("mode,grad,sharding,ckpt", [
    ("full", "cpu_reduce", "rank", True),
    ("full", "gpu_reduce", "rank", True),
    ("shard", "gpu_reduce", "rank", False),
    ("shard", "cpu_reduce", "rank", True),
    ("full", "gpu_reduce", "rank0", True),
])
def test_two_rank_engine_matches_oracle(tmp_path, mode, grad, sharding, ckpt):
    world, steps = 2, 3
    out = str(tmp_path / "res.pt")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=run_engine, args=(r, world, port, mode, grad, sharding, steps, out, ckpt))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = [f for f in os.listdir(tmp_path) if ".err" in f]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    assert all(p.exitcode == 0 for p in procs)
    res0 = torch.load(out)
    res1 = torch.load(out + ".1")
    oracle_losses, oracle_params = _oracle(world, steps)
    for s in range(steps):
        assert abs(res0["losses"][s] - oracle_losses[s][0]) < 1e-4
        assert abs(res1["losses"][s] - oracle_losses[s][1]) < 1e-4
    for n, p in oracle_params.items():
        d = (res0["master"][n].view(p.shape) - p.detach()).abs()
        assert (d > 1e-4).float().mean().item() < 1e-3, n
        assert d.max().item() < 3 * 2 * 1e-3, n



@pytest.mark.parametrize("world,mode,grad", [(4, "full", "gpu_reduce"), (4, "full", "cpu_reduce"),
                                             (8, "full", "gpu_reduce"), (8, "shard", "gpu_reduce")])
def test_many_rank_engine_matches_oracle(tmp_path, world, mode, grad):
    """Four and eight ranks (up to seven shard boundaries per layer, the
    rank count of one 8-GPU node) stay on the oracle's trajectory and
    finite."""
    steps = 4
    out = str(tmp_path / "res.pt")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=run_engine, args=(r, world, port, mode, grad, "rank", steps, out, True))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=400)
    errs = [f for f in os.listdir(tmp_path) if ".err" in f]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    assert all(p.exitcode == 0 for p in procs)
    res = [torch.load(out)] + [torch.load(out + f".{r}") for r in range(1, world)]
    oracle_losses, oracle_params = _oracle(world, steps)
    for s in range(steps):
        for r in range(world):
            assert abs(res[r]["losses"][s] - oracle_losses[s][r]) < 1e-4, (s, r)
    for n, p in oracle_params.items():
        m = res[0]["master"][n].view(p.shape)
        assert torch.isfinite(m).all(), n
        d = (m - p.detach()).abs()
        assert (d > 1e-4).float().mean().item() < 1e-3, n
        assert d.max().item() < steps * 2 * 1e-3, n


@pytest.mark.parametrize("mode,grad,sharding", [("full", "cpu_reduce", "rank"), ("shard", "gpu_reduce", "rank"),
                                                ("full", "gpu_reduce", "rank0")])
def test_two_rank_exact_grad_clip_matches_oracle(tmp_path, mode, grad, sharding):
    """exact_grad_clip: the mean gradient over both ranks is clipped to the
    global norm before any update, as clip_grad_norm_ + AdamW.step.  A large
    eps makes Adam's step proportional to the gradient, so an unclipped (or
    wrongly scaled) update lands far from the oracle."""
    world, steps, clip, eps = 2, 3, 0.05, 1e-2
    out = str(tmp_path / "res.pt")
    port = _free_port()
    ctx = mp.get_context("spawn")
    extra = {"exact_grad_clip": True, "clip_grad_norm": clip, "adam_eps": eps}
    procs = [ctx.Process(target=run_engine, args=(r, world, port, mode, grad, sharding, steps, out, True, extra))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = [f for f in os.listdir(tmp_path) if ".err" in f]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    res0 = torch.load(out)
    oracle_losses, oracle_params, norms = _oracle(world, steps, clip=clip, eps=eps)
    _, unclipped = _oracle(world, steps, eps=eps)
    assert norms[-1] > 10 * clip  # the clip was active
    assert abs(res0["grad_norm"] - norms[-1]) < 1e-4 * norms[-1]
    for s in range(steps):
        assert abs(res0["losses"][s] - oracle_losses[s][0]) < 1e-4
    far = 0.0
    for n, p in oracle_params.items():
        m = res0["master"][n].view(p.shape)
        assert (m - p.detach()).abs().max().item() < 1e-5, n
        far = max(far, (m - unclipped[n].detach()).abs().max().item())
    assert far > 1e-4  # the test tells a clipped run from an unclipped one
