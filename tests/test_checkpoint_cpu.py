"""save_pretrained writes a directory HF transformers loads with identical
outputs; save_state/load_state resume is bit-exact, also on another world
size."""
import pytest
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


def _run_ranks(world, sharding, load_dir, save_dir, steps, tmp_path):
    import os
    import socket

    import torch.multiprocessing as mp

    from tests._dist_worker import run_state

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    err = str(tmp_path / f"state_{world}")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=run_state, args=(r, world, port, sharding, load_dir, save_dir, steps, err))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = [f for f in os.listdir(tmp_path) if ".err" in f]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    assert all(p.exitcode == 0 for p in procs)


def _full_optimizer_state(directory, layer, world):
    import os

    parts = []
    for r in range(world):
        path = os.path.join(directory, f"optim_rank{r}_layer_{layer}.pt")
        if os.path.exists(path):
            sd = torch.load(path)
            parts.append((int(sd["shard"][0]), sd["exp_avg"], sd["exp_avg_sq"], int(sd["step"])))
    parts.sort(key=lambda x: x[0])
    return (torch.cat([p[1] for p in parts]), torch.cat([p[2] for p in parts]), {p[3] for p in parts})


@pytest.mark.parametrize("world_a,world_b,sharding_b", [(2, 1, "rank"), (2, 4, "rank"), (2, 2, "rank0")])
def test_state_saved_at_one_world_size_resumes_at_another(tmp_path, world_a, world_b, sharding_b):
    """Optimizer shards saved by world_a ranks are re-cut for world_b ranks
    (or for a rank-0 optimizer) on load: saving again right after loading
    gives back the same full master and the same full m, v and steps."""
    import os

    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    _run_ranks(world_a, "rank", None, a, 2, tmp_path)
    if world_b == 1:
        torch.manual_seed(0)
        eng = SlideFSDP(LlamaForCausalLM(LlamaConfig.tiny()),
                        SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3))
        eng.load_state(a)
        eng.save_state(b)
        eng.close()
    else:
        _run_ranks(world_b, sharding_b, a, b, 0, tmp_path)
    n_layers = LlamaConfig.tiny().num_hidden_layers + 2
    for i in range(n_layers):
        assert torch.equal(torch.load(os.path.join(a, f"layer_{i}.pt")), torch.load(os.path.join(b, f"layer_{i}.pt")))
        ma, va, sa = _full_optimizer_state(a, i, world_a)
        mb, vb, sb = _full_optimizer_state(b, i, world_b)
        assert torch.equal(ma, mb) and torch.equal(va, vb), i
        assert sa == sb == {2}, (sa, sb)
    if world_b == 1:
        # a missing shard file is reported, not silently zero-filled
        os.remove(os.path.join(a, "optim_rank1_layer_1.pt"))
        torch.manual_seed(0)
        eng = SlideFSDP(LlamaForCausalLM(LlamaConfig.tiny()),
                        SlideFSDPConfig(dtype=torch.float32, device="cpu", lr=1e-3))
        try:
            with pytest.raises(ValueError, match="layer 1: the saved optimizer shards cover"):
                eng.load_state(a)
        finally:
            eng.close()


def test_train_cli_periodic_state_and_resume(tmp_path):
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = str(tmp_path / "out")
    base = [sys.executable, os.path.join(root, "train.py"), "--model-config", "tiny", "--device", "cpu",
            "--batch-size", "2", "--seq-length", "32", "--num-epochs", "1", "--output-dir", out]
    r = subprocess.run(base + ["--max-steps", "6", "--save-state-every", "2"], capture_output=True, text=True,
                       timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    assert open(os.path.join(out, "latest_state")).read() == "state_step6"
    assert sorted(d for d in os.listdir(out) if d.startswith("state_step")) == ["state_step4", "state_step6"]
    r = subprocess.run(base + ["--max-steps", "1", "--resume", out], capture_output=True, text=True,
                       timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "Resumed from" in r.stdout and "state_step6" in r.stdout


def test_train_cli_learning_rate_schedule(tmp_path):
    import importlib.util
    import math
    import os
    import re
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("train_mod", os.path.join(root, "train.py"))
    tm = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tm)
    assert tm.scheduled_lr(1.0, 0, 10, 2, "cosine") == 0.5
    assert tm.scheduled_lr(1.0, 2, 10, 2, "cosine") == 1.0
    assert abs(tm.scheduled_lr(1.0, 6, 10, 2, "cosine") - 0.5) < 1e-12
    assert tm.scheduled_lr(1.0, 6, 10, 2, "linear") == 0.5
    assert tm.scheduled_lr(1.0, 9, 10, 0, "constant") == 1.0
    r = subprocess.run([sys.executable, os.path.join(root, "train.py"), "--model-config", "tiny", "--device", "cpu",
                        "--batch-size", "2", "--seq-length", "32", "--num-epochs", "1", "--max-steps", "4",
                        "--lr", "1e-3", "--lr-scheduler", "cosine", "--warmup-steps", "2",
                        "--output-dir", str(tmp_path / "out")], capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lrs = [float(x) for x in re.findall(r"\| lr ([0-9.e+-]+)", r.stdout)]
    want = [tm.scheduled_lr(1e-3, s, 4, 2, "cosine") for s in range(4)]
    assert len(lrs) == 4 and all(math.isclose(a, b, rel_tol=1e-2) for a, b in zip(lrs, want)), (lrs, want)


def test_train_cli_pins_the_main_thread_to_control_cores(tmp_path):
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cpu = sorted(os.sched_getaffinity(0))[0]
    code = ("import os, sys; sys.argv = ['train.py']; sys.path.insert(0, %r); import train; "
            "train.pin_main_thread(0); print(sorted(os.sched_getaffinity(0)))" % root)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=root,
                       env=dict(os.environ, NUMA_CONTROL_CORES=str(cpu)))
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith(f"[{cpu}]")


def test_train_cli_memory_plan():
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "train.py"), "--model-config", "llama31_8b",
                        "--device", "cpu", "--plan"], capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    plan = json.loads(r.stdout.strip().splitlines()[-1])
    assert abs(plan["params"] - 8.03e9) < 0.01e9 and plan["host_total_gb"] > 100
