"""GPU multi-tensor Adam vs an fp32 PyTorch statement of the same update."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(g, p, m, v, lr, b1, b2, eps, step, mode, bc, wd):
    g, p, m, v = (t.double() for t in (g, p, m, v))
    bc1 = 1 - b1 ** step if bc else 1.0
    bc2 = 1 - b2 ** step if bc else 1.0
    if mode == 0:
        g = g + wd * p
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    upd = (m / bc1) / ((v / bc2).sqrt() + eps)
    if mode == 1:
        upd = upd + wd * p
    return p - lr * upd, m, v


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
@pytest.mark.parametrize("mode", [0, 1])
def test_multi_tensor_adam_matches_reference(dtype, mode):
    from test1_b200.optim.fused_adam import multi_tensor_adam

    torch.manual_seed(0)
    dev = "cuda"
    sizes = [1, 7, 8, 4095, 65537, 300_001]
    big = torch.randn(sum(sizes) + 3, device=dev)
    lists = [[], [], [], []]
    refs = []
    off = 0
    for k, n in enumerate(sizes):
        g = torch.randn(n, device=dev).to(dtype)
        p = torch.randn(n, device=dev).to(dtype)
        m = (torch.randn(n, device=dev) * 0.1).to(dtype)
        v = (torch.rand(n, device=dev) * 0.01).to(dtype)
        if k == 3:  # a view at an odd element offset (scalar path)
            p = big[off + 1: off + 1 + n].to(dtype) if dtype == torch.float32 else p
        off += n
        refs.append(_ref(g, p, m, v, 1e-3, 0.9, 0.999, 1e-8, 3, mode, True, 0.01))
        for l, t in zip(lists, (g, p, m, v)):
            l.append(t)
    noop = torch.zeros(1, dtype=torch.int32, device=dev)
    multi_tensor_adam(1000, noop, lists, 1e-3, 0.9, 0.999, 1e-8, 3, mode, 1, 0.01)
    torch.cuda.synchronize()
    # fp32 arithmetic in the kernel (also for fp64 tensors, as in the
    # reference's functor), including 1 - beta2 formed in fp32 (0.999f makes
    # it 0.00099999 instead of 0.001: a 1.3e-5 relative shift of the v update)
    tol = {torch.float32: 1e-4, torch.float64: 1e-4, torch.bfloat16: 1e-2, torch.float16: 2e-3}[dtype]
    for (rp, rm, rv), p, m, v in zip(refs, lists[1], lists[2], lists[3]):
        for got, want in ((p, rp), (m, rm), (v, rv)):
            err = (got.double() - want).abs() / (want.abs() + 1e-3)
            assert err.max().item() < tol


def test_multi_tensor_adam_many_tensors_and_no_bias_correction():
    from test1_b200.optim.fused_adam import multi_tensor_adam

    torch.manual_seed(1)
    n_t = 450  # three launches of at most 192 tensors
    lists = [[torch.randn(33 + k, device="cuda") for k in range(n_t)] for _ in range(2)]
    lists += [[torch.zeros(33 + k, device="cuda") for k in range(n_t)] for _ in range(2)]
    refs = [_ref(lists[0][k], lists[1][k], lists[2][k], lists[3][k], 1e-2, 0.8, 0.9, 1e-6, 1, 1, False, 0.0)
            for k in range(n_t)]
    multi_tensor_adam(64, torch.zeros(1, dtype=torch.int32, device="cuda"), lists, 1e-2, 0.8, 0.9, 1e-6, 1, 1,
                      0, 0.0)
    for k in range(n_t):
        torch.testing.assert_close(lists[1][k].double(), refs[k][0], rtol=1e-5, atol=1e-6)


def test_fused_adam_optimizer_matches_torch_adamw():
    from test1_b200.optim.fused_adam import FusedAdam

    torch.manual_seed(2)
    a = torch.nn.Linear(257, 129).cuda()
    b = torch.nn.Linear(257, 129).cuda()
    b.load_state_dict(a.state_dict())
    oa = FusedAdam(a.parameters(), lr=1e-3, weight_decay=0.01)
    ob = torch.optim.AdamW(b.parameters(), lr=1e-3, weight_decay=0.01)
    for _ in range(5):
        x = torch.randn(64, 257, device="cuda")
        for mod, opt in ((a, oa), (b, ob)):
            opt.zero_grad()
            mod(x).square().mean().backward()
            opt.step()
    for pa, pb in zip(a.parameters(), b.parameters()):
        torch.testing.assert_close(pa, pb, rtol=1e-5, atol=1e-6)
