"""Weight initialisers (fan-in / fan-out from the tensor's shape, torch
conventions: dim 0 = fan-out, dim 1 (x receptive field) = fan-in).

xavier_uniform U(+-gain*sqrt(6/(fan_in+fan_out))), xavier_normal
N(0, gain^2*2/(fan_in+fan_out)), kaiming/he uniform U(+-gain*sqrt(3/fan)),
kaiming normal N(0, gain^2/fan) with gain sqrt(2) for ReLU, lecun normal
N(0, 1/fan_in), orthogonal (QR of a Gaussian matrix with the sign of R's
diagonal folded in, scaled by gain).

Reference parity: scirs2-neural/src/utils/initializers.rs:221-280
(Initializer::{Xavier, He, LeCun, Orthogonal, Uniform, Normal, Zeros, Ones}).
"""
from __future__ import annotations

import math

import torch


def fans(t: torch.Tensor) -> tuple[int, int]:
    if t.dim() < 2:
        return t.numel(), t.numel()
    rf = t[0][0].numel() if t.dim() > 2 else 1
    return t.shape[1] * rf, t.shape[0] * rf


def calculate_gain(nonlinearity: str, param: float | None = None) -> float:
    return {"linear": 1.0, "sigmoid": 1.0, "tanh": 5.0 / 3, "relu": math.sqrt(2.0),
            "leaky_relu": math.sqrt(2.0 / (1 + (0.01 if param is None else param) ** 2)),
            "selu": 0.75}[nonlinearity]


@torch.no_grad()
def xavier_uniform_(t, gain=1.0, generator=None):
    fi, fo = fans(t)
    a = gain * math.sqrt(6.0 / (fi + fo))
    return t.uniform_(-a, a, generator=generator)


@torch.no_grad()
def xavier_normal_(t, gain=1.0, generator=None):
    fi, fo = fans(t)
    return t.normal_(0.0, gain * math.sqrt(2.0 / (fi + fo)), generator=generator)


@torch.no_grad()
def kaiming_uniform_(t, mode="fan_in", nonlinearity="relu", generator=None):
    fi, fo = fans(t)
    b = calculate_gain(nonlinearity) * math.sqrt(3.0 / (fi if mode == "fan_in" else fo))
    return t.uniform_(-b, b, generator=generator)


@torch.no_grad()
def kaiming_normal_(t, mode="fan_in", nonlinearity="relu", generator=None):
    fi, fo = fans(t)
    return t.normal_(0.0, calculate_gain(nonlinearity) / math.sqrt(fi if mode == "fan_in" else fo),
                     generator=generator)


he_uniform_, he_normal_ = kaiming_uniform_, kaiming_normal_


@torch.no_grad()
def lecun_normal_(t, generator=None):
    return t.normal_(0.0, 1.0 / math.sqrt(fans(t)[0]), generator=generator)


@torch.no_grad()
def orthogonal_(t, gain=1.0, generator=None):
    rows = t.shape[0]
    cols = t.numel() // rows
    a = torch.randn(max(rows, cols), min(rows, cols), generator=generator, dtype=torch.float64)
    q, r = torch.linalg.qr(a)
    q = q * torch.sign(torch.diagonal(r))
    if rows < cols:
        q = q.t()
    return t.copy_((gain * q[:rows, :cols]).reshape(t.shape).to(t.dtype))


def initialize(t: torch.Tensor, name: str, generator=None, **kw):
    fn = {"xavier": xavier_uniform_, "xavier_uniform": xavier_uniform_, "xavier_normal": xavier_normal_,
          "he": kaiming_normal_, "kaiming_uniform": kaiming_uniform_, "kaiming_normal": kaiming_normal_,
          "lecun": lecun_normal_, "orthogonal": orthogonal_}.get(name)
    if name == "zeros":
        return t.zero_()
    if name == "ones":
        return t.fill_(1.0)
    if fn is None:
        raise ValueError(f"unknown initializer {name}")
    return fn(t, generator=generator, **kw)
