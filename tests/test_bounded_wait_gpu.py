"""Bounded device-side waits: a fused kernel whose peer never signals (a flag
nothing sets) must return an error code within its time limit, leaving the
CUDA context usable.  One GPU, one process: no GPU is faulted or hung."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fused_reduce_scatter_times_out_on_missing_peer(cuda_device):
    from test1_b200 import _native

    C = _native.cuda()
    n = 4096
    buf = torch.randn(n, device="cuda").bfloat16()
    pad_mine = torch.zeros(64, dtype=torch.int32, device="cuda")
    pad_ghost = torch.zeros(64, dtype=torch.int32, device="cuda")  # the "peer" never runs
    ptrs = torch.tensor([buf.data_ptr(), buf.data_ptr()], dtype=torch.int64)
    sigs = torch.tensor([pad_mine.data_ptr(), pad_ghost.data_ptr()], dtype=torch.int64)
    out = torch.empty(n // 2, dtype=torch.bfloat16, pin_memory=True)
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.fused_set_peer_wait(2.0)  # default 60 s; a short limit keeps the test short
    try:
        t0 = time.time()
        C.fused_rs_d2h(ptrs, sigs, 0, 2, 0, n // 2, out, 0.5, 1, counter, err)
        torch.cuda.synchronize()
        dt = time.time() - t0
    finally:
        C.fused_set_peer_wait(60.0)
    assert int(err.item()) == 201, "the ready-barrier wait should have expired"
    assert dt < 30
    # the context is still usable
    x = torch.randn(64, 64, device="cuda")
    assert torch.isfinite((x @ x).sum())
