"""Gradient clipping, gradient accumulation and dynamic loss scaling.

  clip_grad_value / clip_grad_norm / clip_grad_global_norm / AdaptiveGradClip
      scirs2-neural/src/training/gradient_clipping.rs:33-429,
      scirs2-autograd/src/gradient_clipping.rs:95-368
  GradientAccumulator   scirs2-autograd/src/gradient_accumulation.rs:63-428
  GradScaler            scirs2-neural/src/training/mixed_precision.rs:98-700

For the flat-buffer optimizers the global-norm clip and the loss-scale
unscale are folded into the fused optimizer launch (max_grad_norm /
grad_multiplier); these helpers serve arbitrary parameter lists.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def _grads(params):
    return [p.grad for p in params if p.grad is not None]


@torch.no_grad()
def clip_grad_value(params, clip_value: float) -> None:
    for g in _grads(params):
        g.clamp_(-clip_value, clip_value)


@torch.no_grad()
def global_norm(params, norm_type: float = 2.0) -> float:
    gs = _grads(params)
    if not gs:
        return 0.0
    if norm_type == float("inf"):
        return float(max(g.abs().max() for g in gs))
    return float(torch.norm(torch.stack([torch.norm(g.float(), norm_type) for g in gs]), norm_type))


@torch.no_grad()
def clip_grad_norm(params, max_norm: float, norm_type: float = 2.0) -> float:
    """Per-tensor norm clipping (each gradient clipped to max_norm)."""
    total = 0.0
    for g in _grads(params):
        n = float(torch.norm(g.float(), norm_type))
        total = max(total, n)
        if n > max_norm:
            g.mul_(max_norm / (n + 1e-6))
    return total


@torch.no_grad()
def clip_grad_global_norm(params, max_norm: float, norm_type: float = 2.0) -> float:
    """Scale all gradients together so their global norm is <= max_norm."""
    n = global_norm(params, norm_type)
    if n > max_norm:
        for g in _grads(params):
            g.mul_(max_norm / (n + 1e-6))
    return n


@dataclass
class AdaptiveGradClip:
    """Adaptive gradient clipping: clip each gradient so that
    ||g|| <= clip_factor * max(||p||, eps) (unit-wise, NFNet-style)."""

    clip_factor: float = 0.01
    eps: float = 1e-3

    @torch.no_grad()
    def __call__(self, params):
        for p in params:
            if p.grad is None:
                continue
            pn = max(float(p.detach().float().norm()), self.eps)
            gn = float(p.grad.float().norm())
            mx = self.clip_factor * pn
            if gn > mx:
                p.grad.mul_(mx / (gn + 1e-6))


class GradientAccumulator:
    """Accumulate gradients over `steps` micro-batches, then average."""

    def __init__(self, steps: int):
        self.steps, self.count, self.buf = steps, 0, None

    @torch.no_grad()
    def accumulate(self, grads):
        if self.buf is None:
            self.buf = [g.detach().clone().float() for g in grads]
        else:
            for b, g in zip(self.buf, grads):
                b.add_(g.float())
        self.count += 1
        return self.count >= self.steps

    def ready(self) -> bool:
        return self.count >= self.steps

    def average(self):
        out = [b / max(self.count, 1) for b in self.buf]
        self.buf, self.count = None, 0
        return out


@dataclass
class MixedPrecisionConfig:
    enabled: bool = True
    initial_loss_scale: float = 65536.0
    growth_factor: float = 2.0
    backoff_factor: float = 0.5
    growth_interval: int = 2000
    min_loss_scale: float = 1.0
    max_loss_scale: float = 2.0**24


class GradScaler:
    """Dynamic loss scaling: scale the loss, unscale gradients, skip steps
    with non-finite gradients, back off on overflow and grow the scale after
    `growth_interval` clean steps."""

    def __init__(self, config: MixedPrecisionConfig | None = None):
        self.config = config or MixedPrecisionConfig()
        self.scale = self.config.initial_loss_scale
        self.growth_tracker = 0
        self.found_inf = False
        self.stats = {"overflows": 0, "steps": 0, "skipped": 0}

    def get_scale(self) -> float:
        return self.scale

    def scale_loss(self, loss):
        return loss * self.scale if self.config.enabled else loss

    @torch.no_grad()
    def unscale_gradients(self, params) -> bool:
        """Divide gradients by the scale; returns True if any is non-finite."""
        if not self.config.enabled:
            return False
        inv = 1.0 / self.scale
        found = False
        for g in _grads(params):
            g.mul_(inv)
            if not torch.isfinite(g).all():
                found = True
        self.found_inf = found
        return found

    def step(self, optimizer, params=None) -> bool:
        """Unscale (when params are given), step unless an overflow was found,
        then update the scale. Returns True if the optimizer stepped."""
        if params is not None:
            self.unscale_gradients(params)
        self.stats["steps"] += 1
        stepped = not self.found_inf
        if stepped:
            optimizer.step()
        else:
            self.stats["skipped"] += 1
        self.update()
        return stepped

    def update(self):
        c = self.config
        if self.found_inf:
            self.stats["overflows"] += 1
            self.scale = max(c.min_loss_scale, self.scale * c.backoff_factor)
            self.growth_tracker = 0
        else:
            self.growth_tracker += 1
            if self.growth_tracker >= c.growth_interval:
                self.scale = min(c.max_loss_scale, self.scale * c.growth_factor)
                self.growth_tracker = 0
        self.found_inf = False
