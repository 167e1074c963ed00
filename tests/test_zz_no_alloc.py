"""GPU test of t1_rmsnorm_bwd_noalloc, the allocation-free RMSNorm backward
(no counterpart in the reference).

Callers that cannot allocate device memory (custom arenas, allocation-free
loops, C programs without PyTorch's allocator) use this exported C symbol.
The test calls it through ctypes, twice in a row with different inputs, and
compares dx and dw with the regular binding `rmsnorm_bwd`, which allocates
its outputs and workspace through PyTorch.  It also checks that the call
leaves PyTorch's allocator statistics untouched.  The file is named so that
pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from test1_b200 import _native

    mod = _native.cuda()
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.t1_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _call(fn, dy, x, w, rstd, resid, dx, dw):
    T, H = x.shape
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
              resid.data_ptr() if resid is not None else None, dx.data_ptr(), dw.data_ptr(),
              T, H, stream)


@pytest.mark.parametrize("T,H", [(1024, 4096), (77, 8192), (5, 256)])
def test_noalloc_matches_regular_binding(T, H, cuda_device):
    from test1_b200.ops import native

    fn = _lib()
    g = torch.Generator(device="cuda").manual_seed(T + H)
    for call in range(2):  # the shared scratch keeps the previous call's contents
        x = (torch.randn(T, H, device="cuda", generator=g) * (call + 1)).bfloat16()
        w = (torch.rand(H, device="cuda", generator=g) + 0.5).bfloat16()
        dy = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        resid = torch.randn(T, H, device="cuda", generator=g).bfloat16() if call == 0 else None
        _, rstd = native.rmsnorm_fwd(x, w, 1e-5)
        dx_ref, dw_ref = native.rmsnorm_bwd(dy, x, w, rstd, resid)
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        torch.cuda.synchronize()
        before = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        rc = _call(fn, dy, x, w, rstd, resid, dx, dw)
        torch.cuda.synchronize()
        after = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        assert rc == 0, f"t1_rmsnorm_bwd_noalloc returned {rc}"
        assert after == before, "the entry point allocated through PyTorch"
        assert _rel(dx, dx_ref) < 5e-3
        assert _rel(dw, dw_ref) < 5e-3


def test_noalloc_rejects_oversized_hidden(cuda_device):
    fn = _lib()
    H = 8200
    x = torch.zeros(2, H, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(H, device="cuda", dtype=torch.bfloat16)
    rstd = torch.zeros(2, device="cuda")
    out = torch.empty_like(x)
    dw = torch.empty_like(w)
    assert _call(fn, x, x, w, rstd, None, out, dw) == 2
    assert _call(fn, x[:, :12], x[:, :12], w[:12], rstd, None, out, dw) == 1  # H % 8 != 0
