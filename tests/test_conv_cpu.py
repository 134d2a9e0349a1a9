"""Convolution / pooling pipeline semantics on the CPU: the im2col / col2im
/ layout helpers and the autograd Functions (through the kernels' CPU
reference paths) reproduce PyTorch's conv2d and pooling, forward and
backward."""
import pytest
import torch
import torch.nn.functional as F

from scirs_b200.ops import functional as FN
from scirs_b200.ops import kernels as K


@pytest.mark.parametrize("C,Cout,k,s,p,d", [(3, 8, 3, 1, 1, 1), (5, 6, 3, 2, 0, 1), (4, 16, 1, 1, 0, 1),
                                            (2, 8, 3, 1, 2, 2)])
def test_conv_fn_matches_torch(C, Cout, k, s, p, d):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, C, 9, 10, generator=g, requires_grad=True)
    w = torch.randn(Cout, C, k, k, generator=g, requires_grad=True)
    b = torch.randn(Cout, generator=g, requires_grad=True)
    y = FN._Conv2dFn.apply(x, w, b, (s, s), (p, p), (d, d))
    yr = F.conv2d(x, w, b, s, p, d)
    assert torch.allclose(y, yr, atol=1e-4)
    gy = torch.randn_like(y)
    gx, gw, gb = torch.autograd.grad(y, (x, w, b), gy)
    rx, rw, rb = torch.autograd.grad(yr, (x, w, b), gy)
    for a, r in ((gx, rx), (gw, rw), (gb, rb)):
        assert torch.allclose(a, r, atol=1e-3), (a - r).abs().max()


@pytest.mark.parametrize("is_max", [True, False])
def test_pool_fn_matches_torch(is_max):
    x = torch.randn(2, 3, 8, 9, generator=torch.Generator().manual_seed(1), requires_grad=True)
    y = FN._Pool2dFn.apply(x, (3, 3), (2, 2), (1, 1), is_max, True)
    yr = F.max_pool2d(x, 3, 2, 1) if is_max else F.avg_pool2d(x, 3, 2, 1)
    assert torch.allclose(y, yr, atol=1e-5)
    gy = torch.randn_like(y)
    (gx,) = torch.autograd.grad(y, x, gy)
    (rx,) = torch.autograd.grad(yr, x, gy)
    assert torch.allclose(gx, rx, atol=1e-5)


def test_rows_layout_roundtrip():
    y = torch.randn(2, 5, 3, 4)
    rows = torch.empty(2 * 12, 8)
    K.conv_nchw_to_rows(y, rows)
    assert torch.equal(rows[:, 5:], torch.zeros(24, 3))
    back = torch.empty_like(y)
    K.conv_rows_to_nchw(rows, back)
    assert torch.equal(back, y)
