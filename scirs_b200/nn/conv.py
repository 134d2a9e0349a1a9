"""Convolution and pooling layers.

  Conv2D                        scirs2-neural/src/layers/conv/conv2d.rs:44-624 (im2col + GEMM,
                                padding modes "valid" / "same" or an explicit amount)
  MaxPool2D / AvgPool2D /
  GlobalAvgPool2D               scirs2-neural/src/layers/conv/pooling.rs
  ResNetBlock                   scirs2-python/tests/test_neural.py:354-415 (API)

On CUDA tensors the convolution runs on the framework's kernels (im2col
kernel -> tcgen05 GEMM with the bias in its epilogue -> NCHW layout kernel;
backward: dgrad GEMM + deterministic col2im gather, fp32 wgrad GEMM, bias
column sums) and pooling on its own max / average kernels, see
scirs_b200/ops/functional.py (conv2d, max_pool2d, avg_pool2d) and
scirs_b200/csrc/conv.cu. On the CPU they use PyTorch (the oracle). Layout
(NCHW) and initialisation follow the reference.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import functional as FN
from .base import Layer
from .layers import BatchNorm


def _pad(padding, k):
    if isinstance(padding, str):
        p = padding.lower()
        if p == "valid":
            return 0
        if p == "same":
            return k // 2
        raise ValueError(f"unknown padding mode {padding}")
    return int(padding)


class Conv2D(Layer):
    def __init__(self, in_channels: int, out_channels: int, kernel_size: int = 3, stride: int = 1, padding=0,
                 bias: bool = True, *, seed=None, dtype=torch.float32, device=None):
        super().__init__()
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        fan_in = in_channels * kernel_size * kernel_size
        bound = 1.0 / math.sqrt(fan_in)
        w = (torch.rand(out_channels, in_channels, kernel_size, kernel_size, generator=g) * 2 - 1) * bound
        self.weight = nn.Parameter(w.to(dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(out_channels, dtype=dtype, device=device)) if bias else None
        self.in_channels, self.out_channels, self.kernel_size = in_channels, out_channels, kernel_size
        self.stride, self.padding = stride, _pad(padding, kernel_size)
        self.padding_mode = padding if isinstance(padding, str) else "explicit"

    def forward(self, x):
        return FN.conv2d(x, self.weight, self.bias, self.stride, self.padding)


class MaxPool2D(Layer):
    def __init__(self, kernel_size=2, stride=None, padding=0):
        super().__init__()
        self.kernel_size, self.stride, self.padding = kernel_size, stride or kernel_size, padding

    def forward(self, x):
        return FN.max_pool2d(x, self.kernel_size, self.stride, self.padding)


class AvgPool2D(Layer):
    def __init__(self, kernel_size=2, stride=None, padding=0):
        super().__init__()
        self.kernel_size, self.stride, self.padding = kernel_size, stride or kernel_size, padding

    def forward(self, x):
        return FN.avg_pool2d(x, self.kernel_size, self.stride, self.padding)


class GlobalAvgPool2D(Layer):
    def forward(self, x):
        return x.mean(dim=(-2, -1))


class ResNetBlock(Layer):
    """conv-bn-relu-conv-bn + (projected) shortcut, relu."""

    def __init__(self, in_channels: int, out_channels: int, stride: int = 1, *, seed=None, dtype=torch.float32,
                 device=None):
        super().__init__()
        kw = dict(dtype=dtype, device=device)
        self.conv1 = Conv2D(in_channels, out_channels, 3, stride, 1, bias=False, seed=seed, **kw)
        self.bn1 = BatchNorm(out_channels, **kw)
        self.conv2 = Conv2D(out_channels, out_channels, 3, 1, 1, bias=False, seed=None if seed is None else seed + 1, **kw)
        self.bn2 = BatchNorm(out_channels, **kw)
        self.proj = None
        if stride != 1 or in_channels != out_channels:
            self.proj = Conv2D(in_channels, out_channels, 1, stride, 0, bias=False, **kw)
            self.proj_bn = BatchNorm(out_channels, **kw)

    def forward(self, x):
        y = torch.relu(self.bn1(self.conv1(x)))
        y = self.bn2(self.conv2(y))
        s = x if self.proj is None else self.proj_bn(self.proj(x))
        return torch.relu(y + s)
