"""Per-phase step tracer on the CPU engine (device brackets fall back to
host clocks without a GPU)."""
import json

import torch

from test1_b200 import SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP


def test_trace_lines_have_every_phase(tmp_path):
    path = tmp_path / "trace.jsonl"
    cfg = LlamaConfig.tiny()
    eng = SlideFSDP(LlamaForCausalLM(cfg, device="meta"),
                    SlideFSDPConfig(dtype=torch.float32, device="cpu", trace_path=str(path)))
    try:
        ids = torch.randint(0, cfg.vocab_size, (2, 16))
        for _ in range(3):
            eng(input_ids=ids, labels=ids)
        eng.wait_for_updates()
    finally:
        eng.close()
    lines = [json.loads(l) for l in path.read_text().splitlines()]
    assert [l["step"] for l in lines] == [1, 2, 3]
    for l in lines:
        for phase in ("fwd", "bwd", "loss", "h2d", "grad_sync"):
            assert phase in l["phase_ms"], (phase, l["phase_ms"])
        assert set(l["layer_ms"]["fwd"]) == {str(i) for i in range(cfg.num_hidden_layers + 1)}
    # optimizer spans are host wall-clock from the update threads
    assert any("adam" in l["phase_ms"] for l in lines)
