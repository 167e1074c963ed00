"""Chunked linear cross-entropy (lm_head GEMM + cross-entropy forward and
backward in token chunks, no [T, V] logits) against the fp32 formula, at the
Llama-3 vocabulary size and an odd token count (the last chunk is one row)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("T,H,chunk", [(513, 256, 128), (64, 512, 4096)])
def test_linear_cross_entropy_matches_fp32(T, H, chunk, cuda_device):
    from test1_b200.ops import native
    from test1_b200.ops import reference as ref

    V = 128256
    g = torch.Generator(device="cuda").manual_seed(T)
    x = (torch.randn(T, H, device="cuda", generator=g)).bfloat16()
    w = (torch.randn(V, H, device="cuda", generator=g) * 0.05).bfloat16()
    targets = torch.randint(0, V, (T,), device="cuda", generator=g)
    targets[::7] = -100  # ignored positions
    dx = torch.empty_like(x)
    dw = torch.full_like(w, float("nan"))  # must be fully written
    loss, count = native.linear_cross_entropy(x, w, targets, dx, dw, chunk)
    dx32 = torch.empty(T, H, device="cuda")
    dw32 = torch.empty(V, H, device="cuda")
    loss32, n32 = ref.linear_cross_entropy(x.float(), w.float(), targets, dx32, dw32, 128)
    torch.cuda.synchronize()
    assert int(count.item()) == n32 == int((targets != -100).sum())
    assert abs(float(loss) - float(loss32)) < 2e-3 * float(loss32)
    assert bool(torch.isfinite(dw.float()).all())
    assert _rel(dx, dx32) < 2e-2
    assert _rel(dw, dw32) < 2e-2
    assert native.gemm_error() == 0


def test_output_layer_chunked_equals_unchunked(cuda_device):
    """The output layer's chunked path gives the loss and gradients of the
    unchunked one (full logits)."""
    from types import SimpleNamespace

    import torch.nn as nn

    from test1_b200.slide_fsdp import OutputLayer

    T, H, V = 1000, 256, 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    norm = nn.Module()
    norm.weight = nn.Parameter((torch.rand(H, device="cuda", generator=g) + 0.5).bfloat16())
    head = nn.Module()
    head.weight = nn.Parameter((torch.randn(V, H, device="cuda", generator=g) * 0.05).bfloat16())
    h = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    ctx = SimpleNamespace(targets=torch.randint(0, V, (T,), device="cuda", generator=g))
    outs = []
    for chunk in (0, 256):
        layer = OutputLayer(norm, head, 1e-5, chunk)
        for p in layer.parameters():
            p.grad = None
        loss, dh = layer.loss_and_grad(h, ctx)
        outs.append((float(loss), dh.clone(), head.weight.grad.clone(), norm.weight.grad.clone()))
    (l0, dh0, gw0, gn0), (l1, dh1, gw1, gn1) = outs
    assert abs(l0 - l1) < 1e-3 * abs(l0)
    assert _rel(dh1, dh0) < 2e-2 and _rel(gw1, gw0) < 2e-2 and _rel(gn1, gn0) < 2e-2
