"""Config validation/round trip, shard math, datasets, FLOPs metric, NUMA
placement on a fake sysfs, split-plane relayout."""
import json
import os

import pytest
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.runtime.layer_state import shard_bounds, shard_size
from test1_b200.runtime.numa import parse_cpulist, plan
from test1_b200.utils.datasets import DummyDataset, UniformTokens
from test1_b200.utils.metric import calculate_flops_per_batch
from test1_b200.utils.param_reuse import fp32_to_split_planes_, split_planes_to_fp32_


def test_config_defaults_and_validation():
    c = SlideFSDPConfig(device="cpu")
    assert c.param_transfer_mode == "full" and c.grad_sync_mode == "gpu_reduce"
    assert c.gpu_buffer_pool_size == 2 and c.adam_betas == (0.9, 0.999)
    with pytest.raises(ValueError, match="param_transfer_mode must be 'full' or 'shard'"):
        SlideFSDPConfig(device="cpu", param_transfer_mode="x")
    with pytest.raises(ValueError, match="grad_sync_mode must be"):
        SlideFSDPConfig(device="cpu", grad_sync_mode="x")
    with pytest.raises(ValueError, match="ac_offload_mode must be"):
        SlideFSDPConfig(device="cpu", ac_offload_mode="disk")
    with pytest.raises(ValueError):
        SlideFSDPConfig(device="cpu", dtype=torch.int8)


def test_config_device_from_local_rank(monkeypatch):
    monkeypatch.setenv("LOCAL_RANK", "3")
    assert SlideFSDPConfig().device == torch.device("cuda", 3)


def test_config_dict_round_trip():
    c = SlideFSDPConfig.from_dict({"dtype": "fp16", "device": "cpu", "adam_betas": [0.8, 0.9],
                                   "param_transfer_mode": "shard", "unknown_key": 1})
    assert c.dtype == torch.float16 and c.adam_betas == (0.8, 0.9) and c.param_transfer_mode == "shard"
    d = c.to_dict()
    assert d["dtype"] == "float16" and d["device"] == "cpu"
    c2 = SlideFSDPConfig.from_dict(json.loads(json.dumps(d)))
    assert c2.to_dict() == d


@pytest.mark.parametrize("P,N", [(1, 2), (100, 3), (218112000, 8), (64 * 7 + 5, 4), (10, 8)])
def test_shard_bounds_cover_exactly(P, N):
    covered = []
    for r in range(N):
        s, e = shard_bounds(P, N, r)
        assert (s % 64 == 0 or s == P) and e <= P and s <= e
        covered.extend(range(s, e)) if P < 10000 else covered.append((s, e))
    if P < 10000:
        assert covered == list(range(P))
    assert shard_size(P, N) * N >= P


def test_dummy_dataset_semantics():
    ds = DummyDataset(size=8, max_length=128, vocab_size=500)
    for i in range(8):
        s = ds[i]
        ids, mask, labels = s["input_ids"], s["attention_mask"], s["labels"]
        assert ids.min() >= 1 and ids.max() < 500
        n = int(mask.sum())
        assert 128 // 3 <= n < 127
        assert not mask[n:].any() and mask[:n].all()
        assert (labels[~mask] == -100).all()
        assert (labels[:10] == -100).all()
        assert torch.equal(labels[100:n], ids[100:n]) or n <= 100
    u = UniformTokens(4, 64, 1000)[0]
    assert torch.equal(u["labels"], u["input_ids"]) and u["attention_mask"].all()


def test_flops_metric_llama8b():
    from test1_b200.models.llama import LlamaConfig

    f = calculate_flops_per_batch(LlamaConfig.llama31_8b(), 4, 1024)
    # ~6 * P_nonembed * T + attention + vocab terms for 4096 tokens
    assert 1.8e14 < f < 2.2e14
    assert calculate_flops_per_batch(LlamaConfig.llama31_8b(), 4, 1024, with_recompute=True) > f


def test_numa_plan_fake_sysfs(tmp_path):
    root = tmp_path
    for n, cpus in [(0, "0-7"), (1, "8-15")]:
        d = root / f"sys/devices/system/node/node{n}"
        d.mkdir(parents=True)
        (d / "cpulist").write_text(cpus)
    for c in range(16):
        d = root / f"sys/devices/system/cpu/cpu{c}/topology"
        d.mkdir(parents=True)
        (d / "thread_siblings_list").write_text(str(c))
    buses = ["00000000:11:00.0", "00000000:12:00.0", "00000000:91:00.0", "00000000:92:00.0"]
    for b, node in zip(buses, [0, 0, 1, 1]):
        d = root / f"sys/bus/pci/devices/{b[4:].lower()}"
        d.mkdir(parents=True)
        (d / "numa_node").write_text(str(node))
    allowed = list(range(16))
    p0 = plan(0, 4, 0, allowed, 1, str(root), buses)
    p1 = plan(1, 4, 1, allowed, 1, str(root), buses)
    p2 = plan(2, 4, 2, allowed, 1, str(root), buses)
    assert p0["NUMA_NODE"] == "0" and p2["NUMA_NODE"] == "1"
    assert parse_cpulist(p0["NUMA_CONTROL_CORES"]) == [0]
    assert parse_cpulist(p0["NUMA_CPU_ADAM_CORES"]) == [1, 2, 3]
    assert parse_cpulist(p1["NUMA_CPU_ADAM_CORES"]) == [5, 6, 7]
    assert parse_cpulist(p2["NUMA_CONTROL_CORES"]) == [8]
    a = set(parse_cpulist(p0["NUMA_CPU_ADAM_CORES"])) | set(parse_cpulist(p0["NUMA_CONTROL_CORES"]))
    b = set(parse_cpulist(p1["NUMA_CPU_ADAM_CORES"])) | set(parse_cpulist(p1["NUMA_CONTROL_CORES"]))
    assert not (a & b)


def test_split_planes_round_trip():
    x = torch.randn(1000) * 10
    orig = x.clone()
    bf = fp32_to_split_planes_(x)
    assert (bf.float() - orig).abs().max() <= orig.abs().max() * 2 ** -8
    split_planes_to_fp32_(x)
    assert torch.equal(x, orig)


def test_native_loader_selects_the_bounds_checked_build(monkeypatch):
    from test1_b200 import _native

    seen = []
    monkeypatch.setattr(_native, "_load", lambda name: seen.append(name) or name)
    monkeypatch.setenv("T1_BOUNDS_CHECK", "1")
    assert _native.cuda() == "_cuda_checked"
    monkeypatch.setenv("T1_BOUNDS_CHECK", "0")
    assert _native.cuda() == "_cuda"


def test_bench_presets_follow_host_ram():
    import importlib.util
    import os

    spec = importlib.util.spec_from_file_location(
        "bench_mod", os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    small = bench.baseline_preset(4, 512 * 2**30)
    assert small["master_layout"] == "bf16" and small["state_dtype"] == "bf16"
    big = bench.baseline_preset(4, 2 * 10**12)
    assert big["master_layout"] == "split" and big["state_dtype"] == "fp32"
    assert bench.baseline_preset(3, 0)["seq"] == 4096 and bench.baseline_preset(2, 0) == {}
    assert bench.host_ram_bytes() > 0


def test_host_traffic_model():
    import importlib.util
    import os

    spec = importlib.util.spec_from_file_location(
        "htm", os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "benchmark",
                            "host_traffic_model.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.bytes_per_param(1, "full") == 32.0
    assert m.bytes_per_param(8, "full") == 26 + 32 + 2
    assert m.bytes_per_param(8, "shard") == 32.0
    rows = m.predict(8.03e9, 190.0, 4096, gpus=(1, 2))
    assert [r["mode"] for r in rows] == ["full", "full", "shard"]
    assert abs(rows[0]["step_s"] - 32 * 8.03e9 / 190e9) < 1e-3


def test_bench_line_carries_the_contract_fields():
    import importlib.util
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_line", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    argv, sys.argv = sys.argv, ["bench.py", "--steps", "4", "--warmup", "3"]
    try:
        args = bench.parse_args()
    finally:
        sys.argv = argv
    res = {"dev_ms": 4 * 1480.0, "clocks": {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []},
           "e2e": {"value": 2700.0, "unit": "tokens/s", "h2d_bytes_per_step": 32768, "d2h_bytes_per_step": 4},
           "launches": 4600, "init_s": 12.0}
    line = bench.make_line(args, 8, res)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "clocks", "e2e", "gpu_launches"):
        assert k in line, k
    assert line["metric"] == bench.METRIC and line["n_gpus"] == 8 and line["scaling"] == "weak"
    assert abs(line["value"] - 8 * 4 * 1024 * 4 / (4 * 1.48)) < 0.01  # whole-job tokens/s
    assert line["ms_per_step"] == 1480.0 and line["higher_is_better"] is True
    for k in ("model", "global_batch", "seq_len", "parallelism"):
        assert k in line["config"], k
    assert line["config"]["global_batch"] == 32 and line["config"]["parallelism"] == "dp8"
    assert line["gpu_launches"] == 4600 and line["detail"]["init_s"] == 12.0


def test_bench_clock_records_merge_over_gpus(monkeypatch):
    import importlib.util
    import os

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_clk", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    recs = [{"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 10},
            {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 9}]

    def fake_gather(out, obj):
        out[:] = recs

    monkeypatch.setattr(dist, "all_gather_object", fake_gather)
    m = bench.merge_clocks(recs[0], 2)
    assert m["sm_mhz"] == 1800.0 and m["reasons"] == ["sw_power_cap"] and m["samples"] == 19
    assert m["per_gpu"] == recs
    assert bench.merge_clocks(recs[0], 1) is recs[0]


def test_clock_sampler_picks_its_gpu_by_bus_id():
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_cs", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    table = "0, 00000000:18:00.0\n3, 00000000:1B:00.0\n"
    pick = bench.ClockSampler.smi_index
    assert pick(0, (0, 0x1B, 0), table) == 3  # CUDA device 0 is nvidia-smi GPU 3
    assert pick(1, (0, 0x99, 0), table) == 1  # unknown bus: the CUDA index
    assert pick(2, None, table) == 2 and pick(2, (0, 0x18, 0), "") == 2


def test_bench_flags_non_finite_losses():
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_fin", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench.all_finite([12.5, 11.9, 11.0], 1)
    assert not bench.all_finite([12.5, float("nan")], 1)
    assert not bench.all_finite([float("inf")], 1)
    assert bench.gather_per_rank({"h2d_gb_per_step": 1.0, "losses": [1.0]}, 1) == [{"h2d_gb_per_step": 1.0}]
