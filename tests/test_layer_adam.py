"""LayerAdam host kernel vs a float64 PyTorch restatement of the update."""
import math

import pytest
import torch

from test1_b200 import _native
from test1_b200.optim import LayerAdam, reference_adamw_

LEVELS = ["scalar", "avx2", "avx512"]


def _supported(level):
    h = _native.host()
    cur = h.simd_level()
    try:
        h.set_simd_level(level)
        return True
    except RuntimeError:
        return False
    finally:
        try:
            h.set_simd_level(cur)
        except RuntimeError:
            pass


@pytest.fixture(params=LEVELS)
def simd(request):
    h = _native.host()
    if not _supported(request.param):
        pytest.skip(f"CPU lacks {request.param}")
    best = h.simd_level()
    h.set_simd_level(request.param)
    yield request.param
    # restore the widest level
    for lvl in reversed(LEVELS):
        try:
            h.set_simd_level(lvl)
            break
        except RuntimeError:
            continue


DTYPES = [
    (torch.float32, torch.float32, torch.float32),
    (torch.float32, torch.bfloat16, torch.float32),
    (torch.float32, torch.float16, torch.float32),
    (torch.bfloat16, torch.bfloat16, torch.float32),
    (torch.bfloat16, torch.bfloat16, torch.bfloat16),
    (torch.float16, torch.float16, torch.float32),
    (torch.float16, torch.float16, torch.float16),
]


def _ulp_tol(dt):
    return {torch.float32: 2e-6, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}[dt]


@pytest.mark.parametrize("pdt,gdt,sdt", DTYPES)
@pytest.mark.parametrize("adamw", [True, False])
@pytest.mark.parametrize("bias_correction", [True, False])
def test_adam_kernel_matches_fp64(simd, pdt, gdt, sdt, adamw, bias_correction):
    h = _native.host()
    torch.manual_seed(1)
    n = 65536 + 77  # exercise vector body, 1-vector loop and scalar tail
    p0 = torch.randn(n, dtype=torch.float64)
    p = p0.to(pdt)
    p64 = p.double()
    m = torch.zeros(n, dtype=sdt)
    v = torch.zeros(n, dtype=sdt)
    m64 = torch.zeros(n, dtype=torch.float64)
    v64 = torch.zeros(n, dtype=torch.float64)
    for step in range(1, 5):
        g = torch.randn(n).to(gdt)
        h.adam_step(p, g, m, v, None, step, 1e-3, 0.9, 0.999, 1e-8, 0.05, bias_correction, adamw, 1.0)
        reference_adamw_(p64, g.double(), m64, v64, step, 1e-3, 0.9, 0.999, 1e-8, 0.05,
                         bias_correction=bias_correction, adamw=adamw)
        if sdt != torch.float32:
            m64.copy_(m.double())
            v64.copy_(v.double())
        if pdt != torch.float32:
            p64.copy_(p.double())
    tol = _ulp_tol(pdt) * (1 + p64.abs())
    assert torch.all((p.double() - p64).abs() <= tol), (p.double() - p64).abs().max()


def test_shadow_is_rne_bf16_of_param(simd):
    h = _native.host()
    torch.manual_seed(2)
    n = 4099
    p = torch.randn(n) * 100
    g = torch.randn(n)
    m = torch.zeros(n)
    v = torch.zeros(n)
    sh = torch.empty(n, dtype=torch.bfloat16)
    h.adam_step(p, g, m, v, sh, 1, 1e-2, 0.9, 0.999, 1e-8, 0.0, True, True, 1.0)
    assert torch.equal(sh, p.bfloat16())


def test_cast_rne_and_nan(simd):
    h = _native.host()
    x = torch.randn(1000) * 1e3
    x[3] = float("nan")
    x[5] = float("inf")
    x[7] = -float("inf")
    x[9] = 1.0 + 2 ** -8  # exact tie -> even
    x[11] = 3.4e38
    out = torch.empty(1000, dtype=torch.bfloat16)
    h.cast_(out, x, 1.0)
    ref = x.bfloat16()
    assert torch.equal(out.view(torch.int16)[~x.isnan()], ref.view(torch.int16)[~x.isnan()])
    assert out.view(torch.int16)[3].item() == 0x7FC0
    out16 = torch.empty(1000, dtype=torch.float16)
    y = torch.randn(1000) * 10
    y[0] = 7e4  # overflows to inf
    y[1] = 1e-7  # subnormal
    h.cast_(out16, y, 1.0)
    assert torch.equal(out16, y.half())


def test_grad_scale_and_zero_grad(simd):
    h = _native.host()
    n = 1000
    p = torch.randn(n)
    g = torch.randn(n)
    pa, pb = p.clone(), p.clone()
    ma, va, mb, vb = (torch.zeros(n) for _ in range(4))
    h.adam_step(pa, g * 0.25, ma, va, None, 1, 1e-3, 0.9, 0.999, 1e-8, 0.01, True, True, 1.0)
    h.adam_step(pb, g, mb, vb, None, 1, 1e-3, 0.9, 0.999, 1e-8, 0.01, True, True, 0.25)
    assert torch.allclose(pa, pb, rtol=1e-6, atol=1e-7)
    pc = p.clone()
    mc, vc = torch.zeros(n), torch.zeros(n)
    h.adam_step(pc, None, mc, vc, None, 1, 1e-3, 0.9, 0.999, 1e-8, 0.01, True, True, 1.0)
    # zero grad: only the decoupled decay acts
    assert torch.allclose(pc, p * (1 - 1e-3 * 0.01), rtol=1e-6, atol=1e-7)


def test_sum_slots_and_sumsq(simd):
    h = _native.host()
    slots = [torch.randn(5000).bfloat16() for _ in range(3)]
    dst = torch.empty(5000)
    h.sum_slots_(dst, slots, 1 / 3)
    ref = sum(s.float() for s in slots) / 3
    assert torch.allclose(dst, ref, atol=1e-6)
    x = torch.randn(100001)
    assert math.isclose(h.sumsq(x), float((x.double() ** 2).sum()), rel_tol=1e-6)


def test_rejects_noncontiguous():
    h = _native.host()
    p = torch.randn(10, 10).t()
    with pytest.raises(RuntimeError, match="contiguous"):
        h.adam_step(p, torch.randn(10, 10), torch.zeros(100), torch.zeros(100), None, 1,
                    1e-3, 0.9, 0.999, 1e-8, 0.0, True, True, 1.0)


def test_layer_adam_api_matches_torch_adamw():
    """LayerAdam.step / step_with_grad_views vs torch.optim.AdamW."""
    torch.manual_seed(3)
    layers = [torch.nn.Linear(33, 17), torch.nn.Linear(17, 5)]
    ref_layers = [torch.nn.Linear(33, 17), torch.nn.Linear(17, 5)]
    for a, b in zip(layers, ref_layers):
        b.load_state_dict(a.state_dict())
    opt = LayerAdam(lr=1e-2, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.1, num_layer=2)
    for i, layer in enumerate(layers):
        assert opt.add_layer_params(i, layer.parameters()) == i
    ref = torch.optim.AdamW([p for l in ref_layers for p in l.parameters()], lr=1e-2,
                            betas=(0.9, 0.99), eps=1e-8, weight_decay=0.1)
    for it in range(5):
        x = torch.randn(8, 33)
        for ls in (layers, ref_layers):
            for p in (q for l in ls for q in l.parameters()):
                p.grad = None
            ls[1](torch.relu(ls[0](x))).square().sum().backward()
        ref.step()
        opt.step(1)
        views = {p: p.grad.clone() for p in layers[0].parameters()}
        opt.step_with_grad_views(0, views)
    for a, b in zip(layers, ref_layers):
        for pa, pb in zip(a.parameters(), b.parameters()):
            assert torch.allclose(pa, pb, atol=1e-5), (pa - pb).abs().max()
    assert opt.param_groups[0]["step"] == 5
    opt.update_learning_rate(5e-3)
    assert all(g["lr"] == 5e-3 for g in opt.param_groups)


def test_layer_adam_flat_and_nvme_offload(tmp_path):
    torch.manual_seed(4)
    n = 10000
    ref_opt = LayerAdam(lr=1e-3, weight_decay=0.01, num_layer=3)
    off_opt = LayerAdam(lr=1e-3, weight_decay=0.01, num_layer=3, nvme_offload_fraction=1.0,
                        offload_dir=str(tmp_path))
    pr = [torch.randn(n) for _ in range(3)]
    po = [p.clone() for p in pr]
    for i in range(3):
        ref_opt.add_flat_layer(i, pr[i])
        off_opt.add_flat_layer(i, po[i])
    for step in range(3):
        for i in reversed(range(3)):
            g = torch.randn(n).bfloat16()
            sh = torch.empty(n, dtype=torch.bfloat16)
            ref_opt.step_flat(i, g)
            off_opt.step_flat(i, g, shadow=sh)
            assert torch.equal(sh, po[i].bfloat16())
    for a, b in zip(pr, po):
        assert torch.equal(a, b)
    off_opt.close()
