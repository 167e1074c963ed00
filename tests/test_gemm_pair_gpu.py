"""CTA-pair (cta_group::2) GEMM vs an fp32 PyTorch product, in all three
operand layouts and with the residual epilogue, at shapes with ragged M, N
and K edges, with both epilogues (register stores: mode 1; shared-memory
staging + TMA stores: mode 2); also checks that the pair path leaves no
error code."""
import pytest
import torch

from test1_b200 import _native
from test1_b200.ops import native

pytestmark = pytest.mark.gpu

SHAPES = [(256, 256, 64), (300, 264, 200), (1000, 776, 1536), (4096, 6144, 4096), (130, 1024, 4096)]


def _rel(a, b):
    return ((a.float() - b).norm() / b.norm().clamp_min(1e-6)).item()


@pytest.fixture(params=[1, 2], ids=["regstore", "tmastore"])
def pair_mode(request):
    C = _native.cuda()
    old = C.gemm_get_mode()
    C.gemm_set_mode(request.param)
    C.gemm_check_error(True)
    yield C
    torch.cuda.synchronize()
    code = C.gemm_check_error(True)
    C.gemm_set_mode(old)
    assert code == 0, f"pair GEMM reported error code {code}"


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_pair_forward(pair_mode, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    assert _rel(native.linear_fwd(x, w), x.float() @ w.float().t()) < 6e-3


@pytest.mark.parametrize("M,N,K", SHAPES[:3])
def test_pair_residual(pair_mode, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16() * 10
    y = native.linear_fwd(x, w, residual=r)
    assert _rel(y, x.float() @ w.float().t() + r.float()) < 6e-3


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_pair_dgrad(pair_mode, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(5)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    assert _rel(native.linear_dgrad(dy, w), dy.float() @ w.float()) < 6e-3


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_pair_wgrad(pair_mode, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(9)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    out = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
    native.linear_wgrad(dy, x, out=out)
    assert _rel(out, dy.float().t() @ x.float()) < 6e-3


@pytest.mark.parametrize("M,N,K", [(300, 264, 200), (1000, 776, 1536)])
def test_pair_wgrad_accumulate(pair_mode, M, N, K):
    """wgrad with the residual epilogue on its own output (C += dy^T x)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    out = (torch.randn(N, K, device="cuda", generator=g) * 4).bfloat16()
    expect = out.float() + dy.float().t() @ x.float()
    native.gemm(dy, x, out, True, True, out)
    assert _rel(out, expect) < 6e-3


@pytest.mark.parametrize("T,S,n_q,n_kv,K", [(4096, 1024, 32, 8, 4096), (300, 100, 4, 2, 512),
                                             (1024, 1024, 32, 8, 4096)])  # last: 96 tiles, stream-K tail
def test_qkv_gemm_with_fused_rope(T, S, n_q, n_kv, K):
    """QKV projection with the rotary embedding applied in the TMA-store
    epilogue (fp32 accumulator rotated before the bf16 rounding) against the
    fp32 product rotated by the reference formula; v columns untouched."""
    from test1_b200.ops import reference as ref

    C = _native.cuda()
    old = C.gemm_get_mode()
    C.gemm_set_mode(2)
    try:
        D = 128
        g = torch.Generator(device="cuda").manual_seed(T + S)
        x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
        w = (torch.randn((n_q + 2 * n_kv) * D, K, device="cuda", generator=g) * 0.05).bfloat16()
        cos, sin = ref.rope_tables(D, S, 500000.0, None, device="cuda")
        out = native.linear_fwd_rope(x, w, cos, sin, S, n_q, n_kv, D)
        expect = ref.rope_qkv_(x.float() @ w.float().t(), n_q, n_kv, D, cos, sin, S)
        assert _rel(out, expect) < 6e-3
        v0 = (n_q + n_kv) * D
        assert _rel(out[:, v0:], expect[:, v0:]) < 6e-3
        torch.cuda.synchronize()
        assert C.gemm_check_error(True) == 0
    finally:
        C.gemm_set_mode(old)


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (512, 512, 2048), (4096, 4096, 14336), (768, 4096, 14336)])
def test_streamk_tail_matches_reference(M, N, K):
    """TMA-store pair GEMM with the stream-K tail (last partial wave split
    along K, partial sums added by the last piece) in the forward, dgrad and
    accumulating wgrad layouts: against the fp32 product, against the same
    GEMM without the split, and twice in a row (the arrival counters are
    reset by the kernel)."""
    C = _native.cuda()
    old = C.gemm_get_mode()
    C.gemm_set_mode(2)
    C.gemm_check_error(True)
    try:
        g = torch.Generator(device="cuda").manual_seed(M + K)
        x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
        w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
        dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
        ref_f = x.float() @ w.float().t()
        outs = []
        for sk in (True, False, True):
            C.gemm_set_streamk(sk)
            y = native.linear_fwd(x, w)
            dx = native.linear_dgrad(dy, w)
            acc = (torch.randn(N, K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1)) * 4).bfloat16()
            expect_acc = acc.float() + dy.float().t() @ x.float()
            native.gemm(dy, x, acc, True, True, acc)
            assert _rel(y, ref_f) < 6e-3
            assert _rel(dx, dy.float() @ w.float()) < 6e-3
            assert _rel(acc, expect_acc) < 6e-3
            outs.append(y)
        # split vs unsplit: same fp32 sums up to the order of addition
        assert _rel(outs[0], outs[1].float()) < 4e-3
        assert torch.equal(outs[0], outs[2])
        torch.cuda.synchronize()
        assert C.gemm_check_error(True) == 0
    finally:
        C.gemm_set_streamk(True)
        C.gemm_set_mode(old)
