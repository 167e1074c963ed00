"""Bounds-checked build of the kernel library (``T1_BUILD_CHECKED=1``
builds ``test1_b200._cuda_checked``; ``T1_BOUNDS_CHECK=1`` selects it).
A training step through the engine with both GEMM and both attention
variants, the multi-tensor Adam and the elementwise kernels at small odd
shapes record no out-of-bounds index; a token id outside the embedding
table, given straight to the kernel, is recorded (and its row skipped)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import os, sys, torch
sys.path.insert(0, os.environ["T1_ROOT"])
from test1_b200 import _native, SlideFSDPConfig
from test1_b200.models.llama import LlamaConfig, LlamaForCausalLM
from test1_b200.slide_fsdp import SlideFSDP
from test1_b200.optim.fused_adam import multi_tensor_adam

C = _native.cuda()
assert C.bounds_checked, "the checked build was not loaded"
C.bounds_errors(True)
dev = torch.device("cuda", 0)
cfg = LlamaConfig(vocab_size=1000, hidden_size=384, intermediate_size=1040, num_hidden_layers=2,
                  num_attention_heads=3, num_key_value_heads=1, rope_theta=500000.0)
eng = SlideFSDP(LlamaForCausalLM(cfg, device="meta"), SlideFSDPConfig(dtype=torch.bfloat16, device=dev))
for gemm_mode, attn_mode in ((1, 1), (0, 0)):
    C.gemm_set_mode(gemm_mode)
    C.attn_set_mode(attn_mode)
    ids = torch.randint(0, cfg.vocab_size, (3, 192))
    loss = float(eng(input_ids=ids, labels=ids).loss)
    assert loss == loss, "nan loss"
    eng.wait_for_updates()
    torch.cuda.synchronize()
    errs = C.bounds_errors(True)
    assert not errs, (gemm_mode, attn_mode, errs)
eng.close()

sizes = [1, 7, 4095, 65537]
lists = [[torch.randn(n, device=dev) for n in sizes] for _ in range(2)]
lists += [[torch.zeros(n, device=dev) for n in sizes] for _ in range(2)]
multi_tensor_adam(1000, torch.zeros(1, dtype=torch.int32, device=dev), lists, 1e-3, 0.9, 0.999, 1e-8,
                  1, 1, 1, 0.01)
torch.cuda.synchronize()
errs = C.bounds_errors(True)
assert not errs, errs

w = torch.randn(64, 128, device=dev).bfloat16()
h = C.embedding_fwd(torch.tensor([3, 64, 5], device=dev), w)
torch.cuda.synchronize()
errs = C.bounds_errors(True)
assert [(e[0], e[2]) for e in errs] == [("embed_ce.cu", 64)], errs
assert torch.equal(h[0], w[3]) and torch.equal(h[2], w[5])
print("bounds-checked build: clean")
"""


def _checked_built() -> bool:
    pkg = os.path.join(ROOT, "test1_b200")
    return any(f.startswith("_cuda_checked") and f.endswith(".so") for f in os.listdir(pkg))


@pytest.mark.skipif(not _checked_built(), reason="bounds-checked build absent (T1_BUILD_CHECKED=1)")
def test_checked_build_records_no_out_of_bounds_access():
    env = dict(os.environ, T1_BOUNDS_CHECK="1", T1_ROOT=ROOT, T1_QUIET="1")
    r = subprocess.run([sys.executable, "-c", SCRIPT], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "clean" in r.stdout
