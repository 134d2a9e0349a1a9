"""Differentiable graph ops (the reference's `tensor_ops`, scirs2-autograd/src/tensor_ops/mod.rs).

`OPS[name](*input_values, **attrs)` evaluates a node; the module-level
functions build nodes. bf16 CUDA matmuls use the framework's tcgen05 GEMM
(via :mod:`scirs_b200.ops.functional`).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..ops import functional as FN
from .graph import Tensor, grad  # noqa: F401


def _mm(a, b):
    if a.dim() == 2 and b.dim() == 2 and a.is_cuda and a.dtype == torch.bfloat16:
        return FN.linear(a, b)
    return a @ b


OPS = {
    "constant": lambda value: value if isinstance(value, torch.Tensor) else torch.as_tensor(value, dtype=torch.float32),
    "zeros": lambda shape: torch.zeros(shape),
    "ones": lambda shape: torch.ones(shape),
    "identity": lambda x: x,
    "add": torch.add,
    "sub": torch.sub,
    "mul": torch.mul,
    "div": torch.div,
    "neg": torch.neg,
    "pow": lambda x, p: x**p,
    "getitem": lambda x, idx: x[idx],
    "matmul": _mm,
    "batch_matmul": torch.matmul,
    "exp": torch.exp,
    "log": torch.log,
    "sqrt": torch.sqrt,
    "square": torch.square,
    "abs": torch.abs,
    "sin": torch.sin,
    "cos": torch.cos,
    "tanh": torch.tanh,
    "sigmoid": torch.sigmoid,
    "relu": torch.relu,
    "leaky_relu": lambda x, alpha: F.leaky_relu(x, alpha),
    "elu": lambda x, alpha: F.elu(x, alpha),
    "gelu": lambda x: F.gelu(x, approximate="tanh"),
    "swish": F.silu,
    "softplus": F.softplus,
    "softmax": lambda x, axis: torch.softmax(x, axis),
    "log_softmax": lambda x, axis: torch.log_softmax(x, axis),
    "reduce_sum": lambda x, axes, keep_dims: x.sum() if axes is None else x.sum(axes, keepdim=keep_dims),
    "reduce_mean": lambda x, axes, keep_dims: x.mean() if axes is None else x.mean(axes, keepdim=keep_dims),
    "reduce_max": lambda x, axes, keep_dims: x.max() if axes is None else x.amax(axes, keepdim=keep_dims),
    "reduce_min": lambda x, axes, keep_dims: x.min() if axes is None else x.amin(axes, keepdim=keep_dims),
    "reduce_prod": lambda x, axes, keep_dims: x.prod() if axes is None else x.prod(axes[0], keepdim=keep_dims),
    "argmax": lambda x, axis: x.argmax(axis),
    "reshape": lambda x, shape: x.reshape(shape),
    "transpose": lambda x, perm: x.permute(*perm) if perm is not None else x.t(),
    "concat": lambda *xs, axis: torch.cat(xs, axis),
    "stack": lambda *xs, axis: torch.stack(xs, axis),
    "slice": lambda x, starts, ends: x[tuple(slice(s, e) for s, e in zip(starts, ends))],
    "expand_dims": lambda x, axis: x.unsqueeze(axis),
    "squeeze": lambda x, axis: x.squeeze(axis),
    "maximum": torch.maximum,
    "minimum": torch.minimum,
    "clip": lambda x, lo, hi: x.clamp(lo, hi),
    "where": lambda c, a, b: torch.where(c.bool(), a, b),
    "one_hot": lambda x, depth: F.one_hot(x.long(), depth).float(),
    "softmax_cross_entropy": lambda logits, t: -(t * torch.log_softmax(logits, -1)).sum(-1),
    "sparse_softmax_cross_entropy": lambda logits, t: F.cross_entropy(logits, t.long().reshape(-1), reduction="none"),
    "sigmoid_cross_entropy": lambda logits, t: F.binary_cross_entropy_with_logits(logits, t, reduction="none"),
    "mse": lambda a, b: ((a - b) ** 2).mean(),
    "conv2d": lambda x, w, stride, padding: F.conv2d(x, w, None, stride, padding),
    "conv2d_transpose": lambda x, w, stride, padding: F.conv_transpose2d(x, w, None, stride, padding),
    "max_pool2d": lambda x, size, stride, padding: F.max_pool2d(x, size, stride, padding),
    "avg_pool2d": lambda x, size, stride, padding: F.avg_pool2d(x, size, stride, padding),
    "batch_norm": lambda x, g, b, eps: F.batch_norm(x, None, None, g, b, True, 0.0, eps),
    "layer_norm": lambda x, g, b, eps: F.layer_norm(x, (x.shape[-1],), g, b, eps),
    "dropout": lambda x, p, train: F.dropout(x, p, train),
    "stop_gradient": lambda x: x.detach(),
    "scale_gradient": lambda x, scale: _ScaleGrad.apply(x, scale),
    "checkpoint": lambda x, fn: torch.utils.checkpoint.checkpoint(fn, x, use_reentrant=False),
    "custom": lambda *xs, fn: fn(*xs),
    "matrix_inverse": torch.linalg.inv,
    "determinant": torch.linalg.det,
    "trace": torch.trace,
    "norm": lambda x, ord_: torch.linalg.norm(x, ord_),
    "svd_values": torch.linalg.svdvals,
    "cholesky": torch.linalg.cholesky,
    "solve": torch.linalg.solve,
    "eigh_values": lambda x: torch.linalg.eigvalsh(x),
}


class _ScaleGrad(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale):
        ctx.scale = scale
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return g * ctx.scale, None


def _n(op, *inputs, **attrs):
    g = next(i.graph for i in inputs if isinstance(i, Tensor))
    ins = [i if isinstance(i, Tensor) else g.constant(i) for i in inputs]
    return Tensor(g, op, ins, attrs)


# ---------------------------------------------------------------------------- builders
def matmul(a, b):
    return _n("matmul", a, b)


def batch_matmul(a, b):
    return _n("batch_matmul", a, b)


def _unary(name):
    def f(x):
        return _n(name, x)

    f.__name__ = name
    return f


for _name in ["exp", "log", "sqrt", "square", "abs", "sin", "cos", "tanh", "sigmoid", "relu", "gelu", "swish",
              "softplus", "stop_gradient", "matrix_inverse", "determinant", "trace", "svd_values", "cholesky",
              "eigh_values"]:
    globals()[_name] = _unary(_name)

detach = globals()["stop_gradient"]


def leaky_relu(x, alpha=0.01):
    return _n("leaky_relu", x, alpha=alpha)


def elu(x, alpha=1.0):
    return _n("elu", x, alpha=alpha)


def softmax(x, axis=-1):
    return _n("softmax", x, axis=axis)


def log_softmax(x, axis=-1):
    return _n("log_softmax", x, axis=axis)


def reduce_sum(x, axes=None, keep_dims=False):
    return _n("reduce_sum", x, axes=axes, keep_dims=keep_dims)


def reduce_mean(x, axes=None, keep_dims=False):
    return _n("reduce_mean", x, axes=axes, keep_dims=keep_dims)


def reduce_max(x, axes=None, keep_dims=False):
    return _n("reduce_max", x, axes=axes, keep_dims=keep_dims)


def reduce_min(x, axes=None, keep_dims=False):
    return _n("reduce_min", x, axes=axes, keep_dims=keep_dims)


def reduce_prod(x, axes=None, keep_dims=False):
    return _n("reduce_prod", x, axes=axes, keep_dims=keep_dims)


def argmax(x, axis=-1):
    return _n("argmax", x, axis=axis)


def reshape(x, shape):
    return _n("reshape", x, shape=tuple(shape))


def transpose(x, perm=None):
    return _n("transpose", x, perm=perm)


def concat(xs, axis=0):
    return _n("concat", *xs, axis=axis)


def stack(xs, axis=0):
    return _n("stack", *xs, axis=axis)


def slice(x, starts, ends):  # noqa: A001
    return _n("slice", x, starts=tuple(starts), ends=tuple(ends))


def expand_dims(x, axis):
    return _n("expand_dims", x, axis=axis)


def squeeze(x, axis):
    return _n("squeeze", x, axis=axis)


def maximum(a, b):
    return _n("maximum", a, b)


def minimum(a, b):
    return _n("minimum", a, b)


def clip(x, lo, hi):
    return _n("clip", x, lo=lo, hi=hi)


def where(c, a, b):
    return _n("where", c, a, b)


def one_hot(x, depth):
    return _n("one_hot", x, depth=depth)


def softmax_cross_entropy(logits, targets):
    return _n("softmax_cross_entropy", logits, targets)


def sparse_softmax_cross_entropy(logits, labels):
    return _n("sparse_softmax_cross_entropy", logits, labels)


def sigmoid_cross_entropy(logits, targets):
    return _n("sigmoid_cross_entropy", logits, targets)


def mean_squared_error(a, b):
    return _n("mse", a, b)


def conv2d(x, w, stride=1, padding=0):
    return _n("conv2d", x, w, stride=stride, padding=padding)


def conv2d_transpose(x, w, stride=1, padding=0):
    return _n("conv2d_transpose", x, w, stride=stride, padding=padding)


def max_pool2d(x, size=2, stride=2, padding=0):
    return _n("max_pool2d", x, size=size, stride=stride, padding=padding)


def avg_pool2d(x, size=2, stride=2, padding=0):
    return _n("avg_pool2d", x, size=size, stride=stride, padding=padding)


def batch_norm(x, gamma, beta, eps=1e-5):
    return _n("batch_norm", x, gamma, beta, eps=eps)


def layer_norm(x, gamma, beta, eps=1e-5):
    return _n("layer_norm", x, gamma, beta, eps=eps)


def dropout(x, p=0.5, train=True):
    return _n("dropout", x, p=p, train=train)


def norm(x, ord_=None):
    return _n("norm", x, ord_=ord_)


def solve(a, b):
    return _n("solve", a, b)


def scale_gradient(x, scale):
    """Identity forward, gradient multiplied by `scale` backward
    (reference: scirs2-autograd/src/custom_gradient.rs)."""
    return _n("scale_gradient", x, scale=scale)


def gradient_reversal(x, lam=1.0):
    return scale_gradient(x, -lam)


def checkpoint(x, fn):
    """Recompute `fn(x)` in the backward pass instead of storing its
    intermediates (reference: tensor_ops/checkpoint_ops.rs:67-606)."""
    return _n("checkpoint", x, fn=fn)


def custom_op(fn, *inputs):
    """Node evaluating an arbitrary differentiable torch function of the inputs."""
    return _n("custom", *inputs, fn=fn)
