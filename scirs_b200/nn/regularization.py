"""Activity regularisation layers: identity in the forward pass that add
l1 * mean|x| + l2 * mean(x^2) of their input to a penalty the training loop
adds to the loss (`layer.loss`, or :func:`regularization_loss` over a
model). Weight penalties: :func:`l1_penalty`, :func:`l2_penalty`.

Reference parity: scirs2-neural/src/layers/regularization.rs:38-460
(ActivityRegularization with optional l1 / l2 factors,
L1ActivityRegularization, L2ActivityRegularization).
"""
from __future__ import annotations

import torch
import torch.nn as nn


class ActivityRegularization(nn.Module):
    def __init__(self, l1_factor: float | None = None, l2_factor: float | None = None, name: str | None = None):
        super().__init__()
        if l1_factor is None and l2_factor is None:
            raise ValueError("at least one of l1_factor / l2_factor is required")
        for f in (l1_factor, l2_factor):
            if f is not None and f < 0:
                raise ValueError("regularisation factors must be non-negative")
        self.l1, self.l2, self.name = l1_factor or 0.0, l2_factor or 0.0, name
        self.loss = torch.zeros(())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        pen = x.new_zeros(())
        if self.l1:
            pen = pen + self.l1 * x.abs().mean()
        if self.l2:
            pen = pen + self.l2 * x.square().mean()
        self.loss = pen
        return x


class L1ActivityRegularization(ActivityRegularization):
    def __init__(self, factor: float, name: str | None = None):
        super().__init__(l1_factor=factor, name=name)


class L2ActivityRegularization(ActivityRegularization):
    def __init__(self, factor: float, name: str | None = None):
        super().__init__(l2_factor=factor, name=name)


def regularization_loss(model: nn.Module) -> torch.Tensor:
    """Sum of the activity penalties recorded by the last forward pass."""
    total = None
    for m in model.modules():
        if isinstance(m, ActivityRegularization):
            total = m.loss if total is None else total + m.loss
    return total if total is not None else torch.zeros(())


def l1_penalty(params, factor: float) -> torch.Tensor:
    return factor * sum(p.abs().sum() for p in params)


def l2_penalty(params, factor: float) -> torch.Tensor:
    return factor * sum(p.square().sum() for p in params)
