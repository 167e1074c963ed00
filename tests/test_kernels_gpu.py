"""sm_100a kernels vs fp32 PyTorch statements of the same ops (ops.reference)."""
import math

import pytest
import torch

from test1_b200.ops import native, reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _gemm_error_clean(cuda_device):
    native.gemm_error(reset=True)
    yield
    torch.cuda.synchronize()
    assert native.gemm_error(reset=True) == 0, "a bounded wait inside the GEMM expired"


GEMM_SHAPES = [(128, 256, 64), (256, 512, 128), (300, 264, 200), (1000, 776, 520), (4096, 6144, 4096)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_forward_layout(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    y = native.linear_fwd(x, w)
    expect = x.float() @ w.float().t()
    assert _rel(y, expect) < 6e-3


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES[:4])
def test_gemm_residual(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16() * 10
    y = native.linear_fwd(x, w, residual=r)
    expect = x.float() @ w.float().t() + r.float()
    assert _rel(y, expect) < 6e-3


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_dgrad_layout(M, N, K):
    # dx [M, K] = dy [M, N] @ W [N, K]
    g = torch.Generator(device="cuda").manual_seed(11)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    dx = native.linear_dgrad(dy, w)
    assert _rel(dx, dy.float() @ w.float()) < 6e-3


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_wgrad_layout(M, N, K):
    # dW [N, K] = dy^T [N, M] @ x [M, K]
    g = torch.Generator(device="cuda").manual_seed(13)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    out = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
    native.linear_wgrad(dy, x, out=out)
    assert _rel(out, dy.float().t() @ x.float()) < 6e-3


def test_gemm_into_strided_output():
    x = torch.randn(256, 512, device="cuda").bfloat16()
    w = torch.randn(384, 512, device="cuda").bfloat16()
    big = torch.zeros(256, 1024, device="cuda", dtype=torch.bfloat16)
    native.gemm(x, w, big[:, 256:640])
    assert _rel(big[:, 256:640], x.float() @ w.float().t()) < 6e-3
    assert big[:, :256].abs().max().item() == 0 and big[:, 640:].abs().max().item() == 0


@pytest.mark.parametrize("T,H", [(7, 256), (1024, 4096), (33, 8192)])
def test_rmsnorm(T, H):
    x = (torch.randn(T, H, device="cuda") * 3).bfloat16()
    w = (torch.rand(H, device="cuda") + 0.5).bfloat16()
    y, rstd = native.rmsnorm_fwd(x, w, 1e-5)
    ye, re = ref.rmsnorm_fwd(x.float(), w.float(), 1e-5)
    assert _rel(y, ye) < 5e-3
    assert torch.allclose(rstd, re, rtol=1e-4)
    dy = torch.randn(T, H, device="cuda").bfloat16()
    res = torch.randn(T, H, device="cuda").bfloat16()
    dx, dw = native.rmsnorm_bwd(dy, x, w, rstd, res)
    dxe, dwe = ref.rmsnorm_bwd(dy.float(), x.float(), w.float(), re, res.float())
    assert _rel(dx, dxe) < 5e-3
    assert _rel(dw, dwe) < 5e-3


def test_rope_qkv_roundtrip():
    T, S, nq, nkv, D = 512, 256, 8, 2, 128
    cos, sin = ref.rope_tables(D, S, 500000.0, {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                "high_freq_factor": 4.0,
                                                "original_max_position_embeddings": 8192}, "cuda")
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda").bfloat16()
    expect = ref.rope_qkv_(qkv.float().clone(), nq, nkv, D, cos, sin, S)
    got = native.rope_qkv_(qkv.clone(), nq, nkv, D, cos, sin, S)
    assert _rel(got, expect) < 5e-3
    back = native.rope_qkv_(got.clone(), nq, nkv, D, cos, sin, S, inverse=True)
    assert _rel(back, qkv) < 1e-2
    assert torch.equal(got[:, (nq + nkv) * D:], qkv[:, (nq + nkv) * D:])  # v untouched


def test_swiglu():
    T, I = 300, 688
    gu = torch.randn(T, 2 * I, device="cuda").bfloat16()
    a = native.swiglu_gu_fwd(gu)
    assert _rel(a, ref.swiglu_gu_fwd(gu.float())) < 5e-3
    da = torch.randn(T, I, device="cuda").bfloat16()
    dgu = native.swiglu_gu_bwd(da, gu)
    assert _rel(dgu, ref.swiglu_gu_bwd(da.float(), gu.float())) < 5e-3


def test_embedding():
    V, H, T = 1000, 256, 777
    w = torch.randn(V, H, device="cuda").bfloat16()
    ids = torch.randint(0, 50, (T,), device="cuda")  # many repeats
    h = native.embedding_fwd(ids, w)
    assert torch.equal(h, w[ids])
    dh = torch.randn(T, H, device="cuda").bfloat16()
    dw = native.embedding_bwd(dh, ids, V)
    dwe = ref.embedding_bwd(dh.float(), ids, V)
    assert _rel(dw, dwe) < 5e-3
    dw2 = native.embedding_bwd(dh, ids, V)
    assert torch.equal(dw, dw2)  # deterministic


@pytest.mark.parametrize("T,V", [(64, 1024), (513, 128256)])
def test_cross_entropy(T, V):
    logits = (torch.randn(T, V, device="cuda") * 2).bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda")
    tgt[::7] = -100
    loss_e, g_e, n = ref.cross_entropy_fwd_bwd(logits.float(), tgt)
    work = logits.clone()
    loss, g, cnt = native.cross_entropy_fwd_bwd(work, tgt)
    assert int(cnt.item()) == n
    assert math.isclose(loss.item(), loss_e.item(), rel_tol=1e-4)
    assert _rel(g, g_e) < 1e-2


@pytest.mark.parametrize("B,S,nq,nkv", [(2, 128, 4, 2), (1, 1024, 32, 8), (2, 256, 8, 8)])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_attention_fwd_bwd(B, S, nq, nkv, mode):
    """Every implementation (0 = mma.sync, 1 = tcgen05 one tile per CTA,
    2 = tcgen05 two tiles per CTA, falling back to 1 when S % 256 != 0) vs
    the fp32 statement."""
    old = native.attn_get_mode()
    native.attn_set_mode(mode)
    try:
        _attention_fwd_bwd_case(B, S, nq, nkv)
    finally:
        native.attn_set_mode(old)


def _attention_fwd_bwd_case(B, S, nq, nkv):
    D = 128
    T = B * S
    g = torch.Generator(device="cuda").manual_seed(S + nq)
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda", generator=g).bfloat16()
    o, lse = native.attention_qkv_fwd(qkv, nq, nkv, D, S)
    oe, lsee = ref.attention_qkv_fwd(qkv.float(), nq, nkv, D, S)
    assert _rel(o, oe) < 1e-2
    assert torch.allclose(lse, lsee, atol=2e-3, rtol=1e-3)
    do = torch.randn(T, nq * D, device="cuda", generator=g).bfloat16()
    dqkv = native.attention_qkv_bwd(do, qkv, o, lse, nq, nkv, D, S)
    dqkve = ref.attention_qkv_bwd(do.float(), qkv.float(), o.float(), lse, nq, nkv, D, S)
    nqd, nkd = nq * D, nkv * D
    assert _rel(dqkv[:, :nqd], dqkve[:, :nqd]) < 2e-2, "dq"
    assert _rel(dqkv[:, nqd:nqd + nkd], dqkve[:, nqd:nqd + nkd]) < 2e-2, "dk"
    assert _rel(dqkv[:, nqd + nkd:], dqkve[:, nqd + nkd:]) < 2e-2, "dv"


@pytest.mark.parametrize("B,S,hq,hkv", [(2, 1024, 4, 2), (1, 192, 2, 1), (2, 320, 8, 2)])
def test_attention_tcgen05_forward_matches_reference(B, S, hq, hkv):
    """tcgen05 forward (TMEM accumulators, P through shared memory) vs the
    fp32 statement, and against the mma.sync forward's outputs."""
    D = 128
    torch.manual_seed(B * S + hq)
    qkv = (torch.randn(B * S, (hq + 2 * hkv) * D, device="cuda") * 0.5).bfloat16()
    old = native.attn_get_mode()
    try:
        native.attn_set_mode(1)
        o, lse = native.attention_qkv_fwd(qkv, hq, hkv, D, S)
        native.attn_set_mode(0)
        o0, lse0 = native.attention_qkv_fwd(qkv, hq, hkv, D, S)
    finally:
        native.attn_set_mode(old)
    torch.cuda.synchronize()
    oe, lsee = ref.attention_qkv_fwd(qkv.float(), hq, hkv, D, S)
    assert _rel(o, oe) < 1e-2
    assert torch.allclose(lse, lsee, atol=2e-3, rtol=1e-3)
    assert _rel(o, o0) < 1e-2
    assert torch.allclose(lse, lse0, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("poly", [0, 1, 2])
@pytest.mark.parametrize("B,S,hq,hkv", [(2, 1024, 4, 2), (1, 256, 2, 1), (1, 2048, 8, 2)])
def test_attention_two_tile_forward(B, S, hq, hkv, poly):
    """Two-tile tcgen05 forward (ping-pong softmax warps, 0/1/2 of every 8
    exponentials on the FMA-pipe polynomial) vs the fp32 statement and the
    one-tile tcgen05 forward."""
    D = 128
    torch.manual_seed(B * S + hq + poly)
    qkv = (torch.randn(B * S, (hq + 2 * hkv) * D, device="cuda") * 0.5).bfloat16()
    old = native.attn_get_mode()
    try:
        native.attn_fwd2_set_poly(poly)
        o2, lse2 = native.attention_fwd_tc2(qkv, hq, hkv, S)
        native.attn_set_mode(1)
        o1, lse1 = native.attention_qkv_fwd(qkv, hq, hkv, D, S)
    finally:
        native.attn_fwd2_set_poly(0)
        native.attn_set_mode(old)
    torch.cuda.synchronize()
    assert native.gemm_error() == 0
    oe, lsee = ref.attention_qkv_fwd(qkv.float(), hq, hkv, D, S)
    assert _rel(o2, oe) < 1e-2
    assert torch.allclose(lse2, lsee, atol=2e-3, rtol=1e-3)
    assert _rel(o2, o1) < 1e-2
    assert torch.allclose(lse2, lse1, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("B,S,nq,nkv", [(2, 256, 4, 2), (1, 320, 8, 2), (2, 1024, 4, 1)])
def test_attention_tcgen05_backward_matches_reference(B, S, nq, nkv):
    D = 128
    T = B * S
    g = torch.Generator(device="cuda").manual_seed(S + nq + 1)
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda", generator=g).bfloat16()
    do = torch.randn(T, nq * D, device="cuda", generator=g).bfloat16()
    old = native.attn_get_mode()
    try:
        native.attn_set_mode(1)
        o, lse = native.attention_qkv_fwd(qkv, nq, nkv, D, S)
        dqkv = native.attention_qkv_bwd(do, qkv, o, lse, nq, nkv, D, S)
    finally:
        native.attn_set_mode(old)
    torch.cuda.synchronize()
    dqkve = ref.attention_qkv_bwd(do.float(), qkv.float(), o.float(), lse, nq, nkv, D, S)
    nqd, nkd = nq * D, nkv * D
    assert _rel(dqkv[:, :nqd], dqkve[:, :nqd]) < 2e-2, "dq"
    assert _rel(dqkv[:, nqd:nqd + nkd], dqkve[:, nqd:nqd + nkd]) < 2e-2, "dk"
    assert _rel(dqkv[:, nqd + nkd:], dqkve[:, nqd + nkd:]) < 2e-2, "dv"


@pytest.mark.parametrize("B,S,nq,nkv", [(2, 256, 4, 2), (1, 320, 8, 2), (2, 1024, 32, 8), (1, 2048, 4, 1)])
def test_attention_pipelined_backward(B, S, nq, nkv):
    """Pipelined tcgen05 backward (double-buffered Q, dQ drained from the dP
    columns while dK runs) vs the fp32 statement and the serial tcgen05
    backward on the same inputs."""
    D = 128
    T = B * S
    g = torch.Generator(device="cuda").manual_seed(7 * S + nq)
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda", generator=g).bfloat16()
    o, lse = native.attention_qkv_fwd(qkv, nq, nkv, D, S)
    do = torch.randn(T, nq * D, device="cuda", generator=g).bfloat16()
    try:
        native.attn_set_bwd_pipelined(True)
        d_pipe = native.attention_qkv_bwd(do, qkv, o, lse, nq, nkv, D, S)
        native.attn_set_bwd_pipelined(False)
        d_ser = native.attention_qkv_bwd(do, qkv, o, lse, nq, nkv, D, S)
    finally:
        native.attn_set_bwd_pipelined(True)
    torch.cuda.synchronize()
    assert native.gemm_error() == 0
    de = ref.attention_qkv_bwd(do.float(), qkv.float(), o.float(), lse, nq, nkv, D, S)
    nqd, nkd = nq * D, nkv * D
    for name, sl in (("dq", slice(0, nqd)), ("dk", slice(nqd, nqd + nkd)), ("dv", slice(nqd + nkd, None))):
        assert _rel(d_pipe[:, sl], de[:, sl]) < 2e-2, name
        assert _rel(d_pipe[:, sl], d_ser[:, sl].float()) < 1e-2, name
