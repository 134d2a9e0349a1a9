"""NumPy-facing API with the contract of the reference's Python bindings.

`import scirs_b200.api as scirs2` gives the surface exercised by the
reference's pytest suite (scirs2-python/tests/test_neural.py and
scirs2-python/tests/test_autograd.py): numpy arrays in and out, method-style
accessors (`layer.in_channels()`, `layer.training(True)`), `loss.compute`,
`optimizer.step(weights, gradients)`, and a small autograd `Tensor`.
Computation is float64 on the CPU by default (the reference's numeric
type); pass `device="cuda"` / `dtype=torch.bfloat16` to the wrapped
:mod:`scirs_b200.nn` layers for the GPU path.
"""
from __future__ import annotations

import contextlib

import numpy as np
import torch

from . import nn as _nn_pkg  # noqa: F401
from .nn import conv as _conv
from .nn import layers as _layers
from .nn import losses as _losses
from .nn.sequential import Sequential as _TorchSequential

_DTYPE = torch.float64


def _t(x, dtype=None):
    if isinstance(x, Tensor):
        return x._t
    if isinstance(x, torch.Tensor):
        return x
    a = np.asarray(x)
    if a.dtype.kind in "iub" and dtype is None:
        return torch.from_numpy(a.astype(np.int64))
    return torch.as_tensor(a, dtype=dtype or _DTYPE)


def _np(t: torch.Tensor):
    return t.detach().cpu().numpy()


# ============================================================================ autograd
_grad_enabled = [True]


@contextlib.contextmanager
def no_grad():
    _grad_enabled.append(False)
    try:
        with torch.no_grad():
            yield
    finally:
        _grad_enabled.pop()


class Tensor:
    """Differentiable array (reference: scirs2-python/src/autograd.rs; the
    graph itself is the framework's autograd over torch)."""

    def __init__(self, data, requires_grad: bool = False):
        t = data._t.detach() if isinstance(data, Tensor) else _t(data).detach().clone()
        if t.dtype != _DTYPE and t.is_floating_point():
            t = t.to(_DTYPE)
        elif not t.is_floating_point():
            t = t.to(_DTYPE)
        self._t = t.requires_grad_(bool(requires_grad) and _grad_enabled[-1])

    @classmethod
    def _wrap(cls, t):
        o = cls.__new__(cls)
        o._t = t
        return o

    # ------------------------------------------------------------ properties
    @property
    def data(self):
        return _np(self._t)

    @property
    def grad(self):
        return None if self._t.grad is None else _np(self._t.grad)

    @property
    def shape(self):
        return tuple(self._t.shape)

    @property
    def requires_grad(self) -> bool:
        return bool(self._t.requires_grad)

    def numpy(self):
        return self.data

    def item(self):
        return float(self._t.item())

    def __repr__(self):
        return f"Tensor({self.data!r}, requires_grad={self.requires_grad})"

    # ------------------------------------------------------------ autograd
    def backward(self, grad=None):
        g = None if grad is None else _t(grad).to(self._t.dtype)
        if g is None and self._t.numel() != 1:
            g = torch.ones_like(self._t)
        self._t.backward(g)

    def zero_grad(self):
        self._t.grad = None

    def detach(self):
        return Tensor._wrap(self._t.detach())

    # ------------------------------------------------------------ ops
    def _bin(self, o, f):
        return Tensor._wrap(f(self._t, _t(o).to(self._t.dtype) if not isinstance(o, (int, float)) else o))

    __add__ = lambda s, o: s._bin(o, torch.add)  # noqa: E731
    __radd__ = __add__
    __sub__ = lambda s, o: s._bin(o, torch.sub)  # noqa: E731
    __rsub__ = lambda s, o: Tensor._wrap(_t(o).to(s._t.dtype) - s._t if not isinstance(o, (int, float)) else o - s._t)  # noqa: E731
    __mul__ = lambda s, o: s._bin(o, torch.mul)  # noqa: E731
    __rmul__ = __mul__
    __truediv__ = lambda s, o: s._bin(o, torch.div)  # noqa: E731
    __rtruediv__ = lambda s, o: Tensor._wrap((o if isinstance(o, (int, float)) else _t(o).to(s._t.dtype)) / s._t)  # noqa: E731
    __matmul__ = lambda s, o: s._bin(o, torch.matmul)  # noqa: E731
    __neg__ = lambda s: Tensor._wrap(-s._t)  # noqa: E731

    def __pow__(self, p):
        return Tensor._wrap(self._t**p)

    def matmul(self, o):
        return self @ o

    def exp(self):
        return Tensor._wrap(self._t.exp())

    def log(self):
        return Tensor._wrap(self._t.log())

    def sqrt(self):
        return Tensor._wrap(self._t.sqrt())

    def sum(self, axis=None):
        return Tensor._wrap(self._t.sum() if axis is None else self._t.sum(axis))

    def mean(self, axis=None):
        return Tensor._wrap(self._t.mean() if axis is None else self._t.mean(axis))

    def relu(self):
        return Tensor._wrap(torch.relu(self._t))

    def sigmoid(self):
        return Tensor._wrap(torch.sigmoid(self._t))

    def tanh(self):
        return Tensor._wrap(torch.tanh(self._t))

    def reshape(self, *shape):
        return Tensor._wrap(self._t.reshape(*shape))

    @property
    def T(self):
        return Tensor._wrap(self._t.t())


def tensor(data, requires_grad=False):
    return Tensor(data, requires_grad)


# ============================================================================ layers
class _NpLayer:
    """Wraps a torch layer; forward takes and returns numpy arrays."""

    _layer: torch.nn.Module

    def forward(self, x):
        with torch.no_grad():
            return _np(self._layer(_t(x)))

    __call__ = forward

    def training(self, flag: bool = True):
        self._layer.train(flag)

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self._layer.parameters())


class Dense(_NpLayer):
    def __init__(self, input_dim, output_dim, activation=None, seed=None):
        self._layer = _layers.Dense(input_dim, output_dim, activation, seed=seed, dtype=_DTYPE)

    def input_dim(self):
        return self._layer.input_dim()

    def output_dim(self):
        return self._layer.output_dim()

    def activation(self):
        return self._layer.activation()


class Conv2D(_NpLayer):
    def __init__(self, in_channels, out_channels, kernel_size=3, stride=1, padding=0, seed=None):
        self._layer = _conv.Conv2D(in_channels, out_channels, kernel_size, stride, padding, seed=seed, dtype=_DTYPE)

    def in_channels(self):
        return self._layer.in_channels

    def out_channels(self):
        return self._layer.out_channels

    def kernel_size(self):
        return self._layer.kernel_size


class MaxPool2D(_NpLayer):
    def __init__(self, kernel_size=2, stride=None, padding=0):
        self._layer = _conv.MaxPool2D(kernel_size, stride, padding)

    def kernel_size(self):
        return self._layer.kernel_size

    def stride(self):
        return self._layer.stride


class AvgPool2D(MaxPool2D):
    def __init__(self, kernel_size=2, stride=None, padding=0):
        self._layer = _conv.AvgPool2D(kernel_size, stride, padding)


class Flatten(_NpLayer):
    def __init__(self):
        self._layer = _layers.Flatten()


class ReLU(_NpLayer):
    def __init__(self):
        self._layer = _layers.ReLU()


class Sigmoid(_NpLayer):
    def __init__(self):
        self._layer = _layers.Sigmoid()


class Tanh(_NpLayer):
    def __init__(self):
        self._layer = _layers.Tanh()


class Softmax(_NpLayer):
    def __init__(self, axis=-1):
        self._layer = _layers.Softmax(axis)


class GELU(_NpLayer):
    def __init__(self):
        self._layer = _layers.GELU()


class Dropout(_NpLayer):
    def __init__(self, rate=0.5):
        self._layer = _layers.Dropout(rate)

    def rate(self):
        return self._layer.p


class BatchNorm(_NpLayer):
    def __init__(self, num_features, momentum=0.1, eps=1e-5):
        self._layer = _layers.BatchNorm(num_features, momentum, eps, dtype=_DTYPE)


class LayerNorm(_NpLayer):
    def __init__(self, normalized_shape, eps=1e-5):
        self._layer = _layers.LayerNorm(normalized_shape, eps, dtype=_DTYPE)


class ResNetBlock(_NpLayer):
    def __init__(self, channels, stride=1, out_channels=None, seed=None):
        self._layer = _conv.ResNetBlock(channels, out_channels or channels, stride, seed=seed, dtype=_DTYPE)


# ============================================================================ losses
class _NpLoss:
    _loss: _losses.Loss

    def compute(self, predictions, targets) -> float:
        with torch.no_grad():
            return float(self._loss(_t(predictions), _t(targets)))

    def gradient(self, predictions, targets):
        return _np(self._loss.backward(_t(predictions), _t(targets)))


class MSELoss(_NpLoss):
    def __init__(self):
        self._loss = _losses.MSELoss()


class CrossEntropyLoss(_NpLoss):
    def __init__(self, from_logits=True):
        self._loss = _losses.CrossEntropyLoss(from_logits=from_logits)


class BinaryCrossEntropyLoss(_NpLoss):
    def __init__(self, from_logits=False):
        self._loss = _losses.BinaryCrossEntropyLoss(from_logits=from_logits)


class HuberLoss(_NpLoss):
    def __init__(self, delta=1.0):
        self._loss = _losses.HuberLoss(delta)


# ============================================================================ optimizers
class _NpOptimizer:
    """`step(weights, gradients) -> updated weights`; state is kept per
    weight array shape/identity, like one optimizer per parameter slot."""

    mode = "sgd"

    def __init__(self, learning_rate=0.01, **hp):
        self.lr, self.hp, self._state = learning_rate, hp, {}

    def _slot(self, w):
        return self._state.setdefault((w.shape, id(w)), {"t": 0, "s1": np.zeros_like(w, dtype=np.float64),
                                                         "s2": np.zeros_like(w, dtype=np.float64)})

    def step(self, weights, gradients):
        from .ops import kernels as K

        w = np.asarray(weights, dtype=np.float64)
        g = np.asarray(gradients, dtype=np.float64)
        st = self._slot(weights)
        st["t"] += 1
        t = st["t"]
        b1 = self.hp.get("beta1", self.hp.get("momentum", self.hp.get("decay_rate", 0.9)))
        b2 = self.hp.get("beta2", 0.999)
        eps = self.hp.get("epsilon", 1e-8)
        wd = self.hp.get("weight_decay", 0.0)
        hp = torch.tensor([self.lr, b1, b2, eps, wd, 1 - self.hp.get("beta1", 0.9) ** t, 1 - b2**t, 1.0, 0.0],
                          dtype=torch.float32)
        p = torch.from_numpy(w.reshape(-1).copy()).float()
        s1 = torch.from_numpy(st["s1"].reshape(-1)).float()
        s2 = torch.from_numpy(st["s2"].reshape(-1)).float()
        K.optim_step(self.mode, p, s1, s2, torch.from_numpy(g.reshape(-1)).float(), None, p.numel(), hp)
        st["s1"], st["s2"] = s1.double().numpy().reshape(w.shape), s2.double().numpy().reshape(w.shape)
        return p.double().numpy().reshape(w.shape)

    def get_learning_rate(self):
        return self.lr

    def set_learning_rate(self, lr):
        self.lr = lr


class SGD(_NpOptimizer):
    mode = "sgd"

    def __init__(self, learning_rate=0.01, momentum=0.0, weight_decay=0.0):
        super().__init__(learning_rate, momentum=momentum, weight_decay=weight_decay)


class Adam(_NpOptimizer):
    mode = "adam"

    def __init__(self, learning_rate=0.001, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.0):
        super().__init__(learning_rate, beta1=beta1, beta2=beta2, epsilon=epsilon, weight_decay=weight_decay)


class AdamW(_NpOptimizer):
    mode = "adamw"

    def __init__(self, learning_rate=0.001, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01):
        super().__init__(learning_rate, beta1=beta1, beta2=beta2, epsilon=epsilon, weight_decay=weight_decay)


class RMSprop(_NpOptimizer):
    mode = "rmsprop"

    def __init__(self, learning_rate=0.001, decay_rate=0.9, epsilon=1e-8, weight_decay=0.0):
        super().__init__(learning_rate, decay_rate=decay_rate, epsilon=epsilon, weight_decay=weight_decay)


class Adagrad(_NpOptimizer):
    mode = "adagrad"

    def __init__(self, learning_rate=0.01, epsilon=1e-10, weight_decay=0.0):
        super().__init__(learning_rate, epsilon=epsilon, weight_decay=weight_decay)


# ============================================================================ model
class Sequential:
    def __init__(self):
        self._m = _TorchSequential()
        self._wrappers = []

    def add(self, layer):
        self._wrappers.append(layer)
        self._m.add(layer._layer if isinstance(layer, _NpLayer) else layer)
        return self

    def num_layers(self) -> int:
        return len(self._wrappers)

    def forward(self, x):
        with torch.no_grad():
            self._m.eval()
            return _np(self._m(_t(x)))

    predict = forward

    def compile(self, optimizer="adam", loss="mse", learning_rate=None, **kw):
        lr = learning_rate if learning_rate is not None else {"sgd": 0.01}.get(str(optimizer).lower(), 1e-3)
        self._m.compile(optimizer, loss, lr, **kw)

    def is_compiled(self) -> bool:
        return self._m.is_compiled()

    def train_step(self, x, y) -> float:
        return self._m.train_batch(_t(x), _t(y))

    def evaluate(self, x, y) -> float:
        return self._m.evaluate(_t(x), _t(y))

    def fit(self, x, y, epochs=10, batch_size=32, validation_split=0.0, verbose=0):
        return self._m.fit(_t(x), _t(y), epochs=epochs, batch_size=batch_size, validation_split=validation_split,
                           verbose=verbose)

    def total_parameters(self) -> int:
        return self._m.total_parameters()

    @property
    def module(self):
        return self._m
