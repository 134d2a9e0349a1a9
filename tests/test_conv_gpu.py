"""Convolution and pooling on the framework's kernels (im2col / col2im /
layout kernels + tcgen05 GEMM; pooling kernels) against PyTorch fp32 on
the same bf16-rounded inputs; Dense+GELU and cross-entropy backward kernels."""
import pytest
import torch
import torch.nn.functional as F

from scirs_b200.ops import functional as FN
from scirs_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("N,C,H,W,Cout,k,s,p,d", [(4, 3, 32, 32, 64, 3, 1, 1, 1), (2, 64, 28, 28, 128, 3, 2, 1, 1),
                                                  (8, 32, 14, 14, 30, 1, 1, 0, 1), (2, 16, 17, 19, 24, 5, 2, 2, 1),
                                                  (2, 8, 16, 16, 16, 3, 1, 2, 2)])
def test_conv2d_kernels_match_fp32(N, C, H, W, Cout, k, s, p, d):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(N, C, H, W, generator=g).cuda().bfloat16().requires_grad_(True)
    w = (torch.randn(Cout, C, k, k, generator=g) / (C * k * k) ** 0.5).cuda().bfloat16().requires_grad_(True)
    b = torch.randn(Cout, generator=g).cuda().bfloat16().requires_grad_(True)
    k0 = K.STATS.launches
    y = FN.conv2d(x, w, b, s, p, d)
    assert K.STATS.launches - k0 == 3  # im2col, GEMM, layout: the native path ran
    xf, wf, bf = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    yr = F.conv2d(xf, wf, bf, s, p, d)
    assert y.shape == yr.shape and _rel(y, yr) < 1e-2
    gy = torch.randn(y.shape, generator=g).cuda().bfloat16()
    gx, gw, gb = torch.autograd.grad(y, (x, w, b), gy)
    rx, rw, rb = torch.autograd.grad(yr, (xf, wf, bf), gy.float())
    assert _rel(gx, rx) < 2e-2 and _rel(gw, rw) < 2e-2 and _rel(gb, rb) < 2e-2
    torch.cuda.synchronize()


@pytest.mark.parametrize("is_max,k,s,p", [(True, 2, 2, 0), (True, 3, 2, 1), (False, 2, 2, 0), (False, 3, 1, 1)])
def test_pooling_kernels_match_fp32(is_max, k, s, p):
    x = torch.randn(4, 16, 23, 20, generator=torch.Generator().manual_seed(1)).cuda().bfloat16().requires_grad_(True)
    y = FN.max_pool2d(x, k, s, p) if is_max else FN.avg_pool2d(x, k, s, p)
    xf = x.detach().float().requires_grad_(True)
    yr = F.max_pool2d(xf, k, s, p) if is_max else F.avg_pool2d(xf, k, s, p)
    assert _rel(y, yr) < 1e-2
    gy = torch.randn_like(y)
    (gx,) = torch.autograd.grad(y, x, gy)
    (rx,) = torch.autograd.grad(yr, xf, gy.float())
    assert _rel(gx, rx) < 2e-2


def test_dense_gelu_and_xent_backward_kernels():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(256, 128, generator=g).cuda().bfloat16().requires_grad_(True)
    w = (torch.randn(128, 256, generator=g) * 0.05).cuda().bfloat16().requires_grad_(True)
    y = FN.linear(x, w, None, activation="gelu")
    logits = y @ (torch.randn(256, 64, generator=g) * 0.05).cuda().bfloat16()
    tgt = torch.randint(0, 64, (256,), generator=g).cuda()
    loss = FN.cross_entropy(logits, tgt)
    gx, gw = torch.autograd.grad(loss, (x, w))
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    # the same projection matrix, regenerated from the seed
    g2 = torch.Generator().manual_seed(2)
    torch.randn(256, 128, generator=g2), torch.randn(128, 256, generator=g2)
    proj = (torch.randn(256, 64, generator=g2) * 0.05).cuda().bfloat16().float()
    lf = F.cross_entropy(F.gelu(xf @ wf, approximate="tanh") @ proj, tgt)
    rx, rw = torch.autograd.grad(lf, (xf, wf))
    assert abs(float(loss) - float(lf)) < 2e-2
    assert _rel(gx, rx) < 3e-2 and _rel(gw, rw) < 3e-2
