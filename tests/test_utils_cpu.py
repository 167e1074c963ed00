"""Utilities without a GPU: the NVML sampler against a fake library,
the module printer, the memory report, sharded HF checkpoint I/O."""
import os
import time
import types

import torch

from test1_b200.utils import checkpoint_io
from test1_b200.utils.gpu_monitor import GPUMonitor
from test1_b200.utils.log_mem import log_memory_stats
from test1_b200.utils.module_utils import module_tree


class _FakeNVML:
    NVML_CLOCK_SM = 1

    def __init__(self):
        self.calls = []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetHandleByIndex(self, i):
        return ("gpu", i)

    def nvmlDeviceGetUtilizationRates(self, h):
        return types.SimpleNamespace(gpu=90, memory=40)

    def nvmlDeviceGetClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetMemoryInfo(self, h):
        return types.SimpleNamespace(used=12e9)

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4  # sw power cap

    # any setter would be a bug: the monitor only reads
    def __getattr__(self, name):
        if name.startswith("nvmlDeviceSet") or name.startswith("nvmlDeviceReset"):
            raise AssertionError(f"GPUMonitor called {name}")
        raise AttributeError(name)


def test_gpu_monitor_samples_and_only_reads():
    nv = _FakeNVML()
    mon = GPUMonitor(device_index=3, interval_s=0.005, nvml=nv).start()
    time.sleep(0.1)
    s = mon.stop()
    assert nv.calls[0] == "init" and nv.calls[-1] == "shutdown"
    assert s["samples"] >= 3 and s["gpu_util_mean"] == 90 and s["sm_mhz_median"] == 1965
    assert abs(s["mem_used_gb_max"] - 12.0) < 1e-9
    assert all(x["reasons"] == 4 for x in mon.samples)


def test_module_tree_and_memory_report():
    m = torch.nn.Sequential(torch.nn.Linear(4, 8), torch.nn.ReLU(), torch.nn.Linear(8, 2))
    text = module_tree(m)
    assert "Linear" in text and "58" in text  # 4*8+8 + 8*2+2 parameters
    assert isinstance(log_memory_stats("x"), str)


def test_sharded_hf_checkpoint_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    tensors = {f"layer.{i}.weight": torch.randn(64, 64, generator=g) for i in range(5)}
    # shards of 2 tensors (64 * 64 * 2 bytes each in bf16)
    checkpoint_io.save_hf_checkpoint(str(tmp_path), {"model_type": "llama"}, tensors, torch.bfloat16,
                                     shard_bytes=2 * 64 * 64 * 2)
    files = sorted(f for f in os.listdir(tmp_path) if f.endswith(".safetensors"))
    assert len(files) == 3 and os.path.exists(tmp_path / "model.safetensors.index.json")
    cfg, back = checkpoint_io.load_hf_checkpoint(str(tmp_path))
    assert cfg["model_type"] == "llama"
    for n, t in tensors.items():
        assert torch.equal(back[n], t.bfloat16()), n


def test_scratch_files_have_no_name_and_round_trip(tmp_path):
    from test1_b200.runtime.scratch_file import ScratchFile

    f = ScratchFile(str(tmp_path))
    data = torch.arange(1 << 20, dtype=torch.int32)
    f.write(memoryview(data.numpy()))
    out = torch.empty_like(data)
    f.read_into(memoryview(out.numpy()))
    assert torch.equal(out, data)
    f.write(memoryview(data[:10].neg().numpy()), offset=8)  # positional, partial overwrite
    f.read_into(memoryview(out.numpy()))
    assert torch.equal(out[2:12], data[:10].neg()) and torch.equal(out[12:], data[12:])
    assert os.listdir(tmp_path) == []  # nothing to leak
    f.close()


def test_memory_plan_matches_the_engine_and_the_8b_layout():
    from test1_b200 import SlideFSDPConfig
    from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
    from test1_b200.slide_fsdp import SlideFSDP
    from test1_b200.utils.memory_plan import plan_memory

    cfg = LlamaConfig.tiny()
    conf = SlideFSDPConfig(dtype=torch.float32, device="cpu")
    eng = SlideFSDP(LlamaForCausalLM(cfg), conf)
    try:
        p = plan_memory(cfg, conf, world=1, batch=2, seq=32)
        assert p["params"] == eng.total_params
        pool_elems = conf.gpu_buffer_pool_size * eng.pool.capacity + eng.big_pool.capacity
        assert abs(p["device_pool_gb_per_gpu"] * 1e9 - pool_elems * 2 * 4) < 1
    finally:
        eng.close()
    big = plan_memory(LlamaConfig.llama31_8b(), SlideFSDPConfig(dtype=torch.bfloat16, device="cpu"), world=1)
    assert abs(big["host_master_gb"] - 32.12) < 0.01 and abs(big["host_optimizer_gb"] - 64.24) < 0.01
    assert abs(big["host_grads_gb"] - 16.06) < 0.01


def test_quickstart_example_runs_on_cpu():
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "examples", "quickstart.py"), "--steps", "2"],
                       capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "step 1: loss" in r.stdout and "model.safetensors" in r.stdout


def test_cpu_adam_benchmark_profiling_modes():
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("cab", os.path.join(root, "benchmark", "cpu_adam_benchmark.py"))
    cab = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cab)
    r = cab.profile_cprofile(10_000, 2, 3, top=5)
    assert r["mode"] == "cprofile" and r["iters"] == 3 and r["min_ms"] > 0
    assert "step" in r["profile"]  # LayerAdam.step shows in the cumulative listing
    p = cab.profile_perf("3B", 1, 1)
    assert p["mode"] == "perf_stat" and ("counters" in p or "unavailable" in p)


def test_reference_linear_cross_entropy_chunks_agree_with_full_logits():
    import torch

    from test1_b200.ops import reference as ref

    T, H, V = 37, 16, 64
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, H, generator=g)
    w = torch.randn(V, H, generator=g) * 0.1
    t = torch.randint(0, V, (T,), generator=g)
    t[::5] = -100
    dx, dw = torch.empty(T, H), torch.empty(V, H)
    loss, n = ref.linear_cross_entropy(x, w, t, dx, dw, 8)
    l_full, dl, n_full = ref.cross_entropy_fwd_bwd(x @ w.t(), t)
    assert n == n_full and abs(float(loss) - float(l_full)) < 1e-5
    assert torch.allclose(dx, dl @ w, atol=1e-6) and torch.allclose(dw, dl.t() @ x, atol=1e-6)


def test_wgrad_in_row_blocks_matches_one_product():
    import torch

    from test1_b200.models.llama import _wgrad_in_chunks

    g = torch.Generator().manual_seed(1)
    dy = torch.randn(64, 1000, generator=g)
    x = torch.randn(64, 48, generator=g)
    out = torch.empty(1000, 48)
    seen = []
    _wgrad_in_chunks(dy, x, out, lambda t: seen.append((t.data_ptr() - out.data_ptr()) // 4 // 48), 3)
    assert torch.allclose(out, dy.t() @ x, atol=1e-4)
    assert seen == [0, 512]  # 256-row aligned blocks: [0, 512), [512, 1000)
