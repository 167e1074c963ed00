"""SlidingCheckpoint around torch.utils.checkpoint on the GPU: tensors saved
by each checkpointed layer go to the pinned host slots (the last layer keeps
them on the device), the backward brings them back, and gradients equal
those of a plain run."""
import pytest
import torch
from torch.utils.checkpoint import checkpoint

from test1_b200.sliding_checkpoint import SlidingCheckpoint, reset_prefetch_state

pytestmark = pytest.mark.gpu


def _layers(n, h):
    torch.manual_seed(0)
    return torch.nn.ModuleList(torch.nn.Sequential(torch.nn.Linear(h, h), torch.nn.GELU()) for _ in range(n)).cuda()


def test_sliding_checkpoint_matches_plain_backward():
    n, h, T = 4, 256, 512
    layers = _layers(n, h)
    x = torch.randn(T, h, device="cuda", requires_grad=True)

    y = x
    for l in layers:
        y = l(y)
    y.square().mean().backward()
    ref_x = x.grad.clone()
    ref_w = [l[0].weight.grad.clone() for l in layers]
    x.grad = None
    for l in layers:
        l.zero_grad(set_to_none=True)

    # slots: the checkpoint saves the layer input (one [T, h] tensor)
    slots = [[torch.empty(T, h, pin_memory=True)] for _ in range(n)]
    reset_prefetch_state()
    y = x
    for i, l in enumerate(layers, start=1):
        with SlidingCheckpoint(layer_idx=i, layer_tensors=slots, is_last_layer=(i == n), no_mask=True,
                               device="cuda:0"):
            y = checkpoint(l, y, use_reentrant=False)
    y.square().mean().backward()
    torch.cuda.synchronize()
    torch.testing.assert_close(x.grad, ref_x)
    for l, w in zip(layers, ref_w):
        torch.testing.assert_close(l[0].weight.grad, w)
    # layers 1..n-1 went through host memory
    assert torch.count_nonzero(slots[0][0]) > 0
