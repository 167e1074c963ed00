"""GPU test of t1_rmsnorm_bwd_noalloc, the allocation-free RMSNorm backward
(no counterpart in the reference).

Callers that cannot allocate device memory (custom arenas, allocation-free
loops, C programs without PyTorch's allocator) use this exported C symbol.
The test calls it through ctypes, twice in a row with different inputs, and
compares dx and dw with the regular binding `rmsnorm_bwd`, which allocates
its outputs and workspace through PyTorch, and with the fp32 formula of
`ops.reference.rmsnorm_bwd`.  It checks that a call leaves PyTorch's
allocator statistics untouched and that the device's free memory
(cudaMemGetInfo) is the same before and after a call, which also catches a
raw cudaMalloc.  The file is named so that pytest collects it last.
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


def _call(fn, dy, x, w, rstd, resid, dx, dw, T=None):
    H = x.shape[1]
    T = x.shape[0] if T is None else T
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
              resid.data_ptr() if resid is not None else None, dx.data_ptr(), dw.data_ptr(),
              T, H, stream)


def _rows(t, T):
    """View of the first T rows; the full buffer is what the C call gets, so
    its pointers stay valid (non-null) when T is 0."""
    return t[:T]


@pytest.mark.parametrize("T,H", [(1024, 4096), (77, 8192), (5, 256), (33, 5120), (0, 1024)])
def test_noalloc_matches_regular_binding(T, H, cuda_device):
    from test1_b200.ops import native
    from test1_b200.ops import reference as ref

    fn = _lib()
    g = torch.Generator(device="cuda").manual_seed(T + H)
    rows = max(T, 1)  # T = 0 still passes valid (unread) row buffers
    for call in range(2):  # the shared scratch keeps the previous call's contents
        xb = (torch.randn(rows, H, device="cuda", generator=g) * (call + 1)).bfloat16()
        w = (torch.rand(H, device="cuda", generator=g) + 0.5).bfloat16()
        dyb = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
        rb = torch.randn(rows, H, device="cuda", generator=g).bfloat16() if call == 0 else None
        x, dy = _rows(xb, T), _rows(dyb, T)
        resid = _rows(rb, T) if rb is not None else None
        if T:
            _, rstd = native.rmsnorm_fwd(x, w, 1e-5)
            dx_ref, dw_ref = native.rmsnorm_bwd(dy, x, w, rstd, resid)
            rstdb = rstd
        else:
            rstdb = torch.zeros(1, device="cuda")
            rstd = rstdb[:0]
            dx_ref, dw_ref = torch.empty_like(x), torch.zeros_like(w)
        # fp32 oracle of the same formula
        dx32, dw32 = ref.rmsnorm_bwd(dy.float(), x.float(), w.float(), rstd,
                                     resid.float() if resid is not None else None)
        dxb = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
        dx = _rows(dxb, T)
        dw = torch.full_like(w, float("nan"))  # must be overwritten, also for T = 0
        torch.cuda.synchronize()
        before = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        free_before = torch.cuda.mem_get_info()[0]
        rc = _call(fn, dyb, xb, w, rstdb, rb, dxb, dw, T)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        after = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        assert rc == 0, f"t1_rmsnorm_bwd_noalloc returned {rc}"
        assert after == before, "the entry point allocated through PyTorch"
        if call == 1:
            # the first call of a process may load the library's module (with
            # its scratch array) lazily; a later call must not change the
            # device's free memory
            assert free_after == free_before, "device free memory changed across the call"
        if T == 0:
            assert bool((dw.float() == 0).all()), "T = 0 must write a zero dw"
            continue
        assert _rel(dx, dx_ref) < 5e-3
        assert _rel(dw, dw_ref) < 5e-3
        assert _rel(dx, dx32) < 5e-3
        assert _rel(dw, dw32) < 5e-3


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
