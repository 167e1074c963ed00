"""Host-memory registration plan of the engine (which ranges each rank's GPU
reads) and the early norm-weight fetch of shard mode, on CPU."""
import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP


def _engine(**kw):
    cfg = LlamaConfig.tiny()
    torch.manual_seed(0)
    return SlideFSDP(LlamaForCausalLM(cfg), SlideFSDPConfig(dtype=torch.bfloat16, device="cpu", **kw))


def test_pin_ranges_cover_every_read_on_page_boundaries_without_overlap():
    eng = _engine()
    try:
        ranges = eng._pin_ranges()
        assert ranges, "full mode reads every layer's bf16 copy"
        prev_end = -1
        for off, n in ranges:
            assert off % 4096 == 0 and n % 4096 == 0 or off + n == eng.shared.nbytes
            assert off > prev_end  # sorted, disjoint, not even touching
            prev_end = off + n
        base = eng.shared.buf.data_ptr()
        for st in eng.layer_states:
            for t in eng.comm.host_read_views(st):
                a = t.data_ptr() - base
                b = a + t.numel() * t.element_size()
                assert any(off <= a and b <= off + n for off, n in ranges), st.idx
        # the split master's low planes are never read by the GPU in full mode
        # (only the page a plane shares with the preceding high plane is pinned)
        lo = eng.stores[1].lo
        a = lo[lo.numel() // 2:].data_ptr() - base
        assert not any(off <= a < off + n for off, n in ranges)
    finally:
        eng.close()


def test_early_weight_is_the_rounded_master():
    eng = _engine()
    try:
        st = eng.layer_states[1]
        w = eng._early_weight(st, "input_layernorm.weight")
        e = next(e for e in st.layout.entries if e.name == "input_layernorm.weight")
        ref = st.store.read_fp32(e.offset, e.offset + e.numel).bfloat16()
        assert w.dtype == torch.bfloat16 and torch.equal(w.cpu(), ref.view(e.shape))
    finally:
        eng.close()


def test_master_shards_get_numa_placement_on_multi_node_hosts(monkeypatch):
    from test1_b200 import _native
    from test1_b200.runtime import numa

    calls = []
    host = _native.host()

    class Spy:
        def __getattr__(self, name):
            return getattr(host, name)

        def numa_bind(self, t, nodes, mode):
            calls.append((t.data_ptr(), t.numel(), tuple(nodes), mode))
            return 0

    monkeypatch.setattr(numa, "numa_nodes", lambda root="/": {0: [0, 1], 1: [2, 3]})
    monkeypatch.setenv("NUMA_NODE", "1")
    monkeypatch.setattr(_native, "host", lambda: Spy())
    eng = _engine()
    try:
        # one preferred placement per plane of every layer's optimizer shard
        assert len(calls) == 2 * eng.num_layers
        assert all(c[2] == (1,) and c[3] == "preferred" for c in calls)
    finally:
        monkeypatch.undo()
        eng.close()
