"""Core layers: Dense, activations, Dropout, Flatten, LayerNorm, BatchNorm,
Embedding, PositionalEmbedding.

Semantics follow the reference (file:line cited per class); bf16 CUDA
tensors run on the sm_100a kernels through :mod:`scirs_b200.ops.functional`.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import functional as FN
from .base import Layer


class Dense(Layer):
    """Fully connected layer y = act(x @ W + b), W stored [input_dim, output_dim].

    Init as the reference: W ~ U(-1, 1) / sqrt(input_dim), b = 0
    (scirs2-neural/src/layers/dense.rs:82-139). Optional fused activation by
    name: relu / sigmoid / tanh / softmax / gelu (gelu is fused into the GEMM
    epilogue on the tensor-core path).
    """

    def __init__(self, input_dim: int, output_dim: int, activation: str | None = None, *, seed: int | None = None,
                 dtype=torch.float32, device=None):
        super().__init__()
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        w = (torch.rand(input_dim, output_dim, generator=g) * 2 - 1) / math.sqrt(input_dim)
        self.weight = nn.Parameter(w.to(dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(output_dim, dtype=dtype, device=device))
        self._in, self._out, self._act = input_dim, output_dim, activation

    def forward(self, x):
        return FN.linear(x, self.weight, self.bias, self._act)

    def input_dim(self) -> int:
        return self._in

    def output_dim(self) -> int:
        return self._out

    def activation(self) -> str | None:
        return self._act


class _Act(Layer):
    fn = None

    def forward(self, x):
        return type(self).fn(x)


class ReLU(_Act):
    fn = staticmethod(torch.relu)


class Sigmoid(_Act):
    fn = staticmethod(torch.sigmoid)


class Tanh(_Act):
    fn = staticmethod(torch.tanh)


class Softmax(Layer):
    def __init__(self, dim: int = -1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.softmax(x, self.dim)


class GELU(Layer):
    """GELU; `fast=True` (default) is the tanh form used throughout the
    framework (reference activations_minimal.rs:57-68), `fast=False` the
    exact erf form."""

    def __init__(self, fast: bool = True):
        super().__init__()
        self.fast = fast

    def forward(self, x):
        return F.gelu(x, approximate="tanh" if self.fast else "none")


class Swish(_Act):
    fn = staticmethod(F.silu)


class Mish(_Act):
    fn = staticmethod(F.mish)


class LeakyReLU(Layer):
    def __init__(self, alpha: float = 0.01):
        super().__init__()
        self.alpha = alpha

    def forward(self, x):
        return F.leaky_relu(x, self.alpha)


class ELU(Layer):
    def __init__(self, alpha: float = 1.0):
        super().__init__()
        self.alpha = alpha

    def forward(self, x):
        return F.elu(x, self.alpha)


class Dropout(Layer):
    """Inverted dropout (scirs2-neural/src/layers/dropout.rs)."""

    def __init__(self, p: float = 0.5):
        super().__init__()
        if not 0 <= p < 1:
            raise ValueError("dropout rate must be in [0, 1)")
        self.p = p

    def forward(self, x):
        return F.dropout(x, self.p, self.training)

    def rate(self) -> float:
        return self.p


class Flatten(Layer):
    def forward(self, x):
        return x.reshape(x.shape[0], -1)


class LayerNorm(Layer):
    """LayerNorm over the last dimension (scirs2-neural/src/layers/normalization.rs:93-260;
    here with the full backward)."""

    def __init__(self, normalized_shape: int, eps: float = 1e-5, dtype=torch.float32, device=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(normalized_shape, dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(normalized_shape, dtype=dtype, device=device))
        self.eps = eps

    def forward(self, x):
        return FN.layer_norm(x, self.weight, self.bias, self.eps)


class BatchNorm(Layer):
    """Batch normalisation over the channel dimension (dim 1), with running
    statistics for inference (scirs2-neural/src/layers/normalization.rs:343)."""

    def __init__(self, num_features: int, momentum: float = 0.1, eps: float = 1e-5, dtype=torch.float32, device=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(num_features, dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(num_features, dtype=dtype, device=device))
        sdt = torch.float32 if dtype in (torch.bfloat16, torch.float16) else dtype
        self.register_buffer("running_mean", torch.zeros(num_features, dtype=sdt, device=device))
        self.register_buffer("running_var", torch.ones(num_features, dtype=sdt, device=device))
        self.momentum, self.eps = momentum, eps

    def forward(self, x):
        return F.batch_norm(x, self.running_mean, self.running_var, self.weight, self.bias, self.training,
                            self.momentum, self.eps)


class Embedding(Layer):
    """Token embedding lookup (scirs2-neural/src/layers/embedding.rs:16-330)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, dtype=torch.float32, device=None, seed=None):
        super().__init__()
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        self.weight = nn.Parameter(torch.randn(num_embeddings, embedding_dim, generator=g).to(dtype=dtype, device=device))

    def forward(self, tok):
        return FN.embedding(tok, self.weight)


class PositionalEmbedding(Layer):
    """Positional embedding: learned table or fixed sinusoidal
    (scirs2-neural/src/layers/embedding.rs:292-661)."""

    def __init__(self, max_len: int, dim: int, learned: bool = False, dtype=torch.float32, device=None):
        super().__init__()
        self.learned = learned
        if learned:
            self.weight = nn.Parameter(torch.randn(max_len, dim, dtype=dtype, device=device) * 0.02)
        else:
            pos = torch.arange(max_len, dtype=torch.float32)[:, None]
            div = torch.exp(torch.arange(0, dim, 2, dtype=torch.float32) * (-math.log(10000.0) / dim))
            pe = torch.zeros(max_len, dim)
            pe[:, 0::2] = torch.sin(pos * div)
            pe[:, 1::2] = torch.cos(pos * div[: dim // 2])
            self.register_buffer("pe", pe.to(dtype=dtype, device=device))

    def forward(self, x):
        S = x.shape[1]
        table = self.weight if self.learned else self.pe
        return x + table[:S].to(x.dtype)
