"""SlidingCheckpoint without a GPU (the reference creates a CUDA stream at
import and cannot run there): saved tensors go to the host slots and the
backward matches a plain run."""
import torch
from torch.utils.checkpoint import checkpoint

from test1_b200.sliding_checkpoint import SlidingCheckpoint, reset_prefetch_state


def test_sliding_checkpoint_on_cpu_matches_plain_backward():
    n, h, T = 3, 32, 16
    torch.manual_seed(0)
    layers = torch.nn.ModuleList(torch.nn.Sequential(torch.nn.Linear(h, h), torch.nn.GELU()) for _ in range(n))
    x = torch.randn(T, h, requires_grad=True)
    y = x
    for l in layers:
        y = l(y)
    y.square().mean().backward()
    ref_x = x.grad.clone()
    ref_w = [l[0].weight.grad.clone() for l in layers]
    x.grad = None
    for l in layers:
        l.zero_grad(set_to_none=True)

    slots = [[torch.empty(T, h)] for _ in range(n)]
    reset_prefetch_state()
    y = x
    for i, l in enumerate(layers, start=1):
        with SlidingCheckpoint(layer_idx=i, layer_tensors=slots, is_last_layer=(i == n), no_mask=True,
                               device="cpu"):
            y = checkpoint(l, y, use_reentrant=False)
    y.square().mean().backward()
    torch.testing.assert_close(x.grad, ref_x)
    for l, w in zip(layers, ref_w):
        torch.testing.assert_close(l[0].weight.grad, w)
    assert torch.count_nonzero(slots[0][0]) > 0  # layer 1's input went through its host slot
