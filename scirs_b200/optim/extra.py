"""Per-tensor optimizers whose update needs whole-tensor statistics (norms,
factored moments): RAdam, LAMB, LARS/LARC, Adafactor, Sophia.

They follow torch.optim's interface (`step`, `zero_grad`, `state_dict`,
param groups) plus the reference's `get_learning_rate` /
`set_learning_rate`, and run on whatever device the parameters live on
(torch foreach/tensor ops; none of them is on a flagship hot path, where the
fused flat optimizer kernel is used).

Update rules (reference scirs2-neural/src/optimizers/):
  RAdam     radam.rs:27-250   Adam with variance rectification
            (rho_inf = 2/(1-beta2) - 1; un-adapted momentum step while
            rho_t <= 4, weight decay added to the gradient). The default
            rectification is the paper's (Liu et al. 2020,
            sqrt((rho-4)(rho-2)rho_inf / ((rho_inf-4)(rho_inf-2)rho)));
            rectification="reference" reproduces radam.rs:209-214,
            ((rho-2)/(rho-4)) * sqrt((rho-2)/rho)
  LAMB      lamb.rs:32-200    u = m_hat/(sqrt(v_hat)+eps) + wd*p;
            trust = ||p||/||u|| (1 when either is 0, optional clamp);
            p -= lr*trust*u
  LARS      lars.rs:31-238    local_lr = eta*||w||/(||g|| + wd*||w|| + eps)
            (LARC: min(local_lr, lr)); v = mu*v + local_lr*(g + wd*w); w -= v
  Adafactor adafactor.rs:44-420  RMS-clipped gradient, beta2_t = 1 - t^-0.8,
            factored row/column second moment for >= 2-D tensors whose dims
            are both >= min_dim_size_to_factor, relative step 1/sqrt(t)
            (>= min lr) unless a fixed lr is given (then a 0.9 EMA of the
            update)
  Sophia    sophia.rs:27-260  m = b1*m + (1-b1)*g;
            h <- b2*h + (1-b2)*(g*z)^2 every `hessian_period` steps
            (z Rademacher, Hutchinson); d = max(rho*h, eps);
            p -= lr*(clamp(m/d, -1, 1)*d + wd*p)
"""
from __future__ import annotations

import math

import torch
from torch.optim import Optimizer


class _LrMixin:
    def get_learning_rate(self) -> float:
        return self.param_groups[0]["lr"]

    def set_learning_rate(self, lr: float) -> None:
        for g in self.param_groups:
            g["lr"] = lr


class RAdam(_LrMixin, Optimizer):
    def __init__(self, params, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, rectification="paper"):
        assert rectification in ("paper", "reference")
        super().__init__(params, dict(lr=lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay))
        self.rectification = rectification

    def _rect(self, rho_t, rho_inf):
        if self.rectification == "reference":
            return (rho_t - 2) / (rho_t - 4) * math.sqrt((rho_t - 2) / rho_t)
        return math.sqrt((rho_t - 4) * (rho_t - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho_t))

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for g in self.param_groups:
            b1, b2 = g["beta1"], g["beta2"]
            rho_inf = 2.0 / (1.0 - b2) - 1.0
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["t"], st["m"], st["v"] = 0, torch.zeros_like(p), torch.zeros_like(p)
                st["t"] += 1
                t = st["t"]
                grad = p.grad if g["weight_decay"] == 0 else p.grad + g["weight_decay"] * p
                st["m"].mul_(b1).add_(grad, alpha=1 - b1)
                st["v"].mul_(b2).addcmul_(grad, grad, value=1 - b2)
                m_hat = st["m"] / (1 - b1 ** t)
                b2t = b2 ** t
                rho_t = rho_inf - 2.0 * t * b2t / (1.0 - b2t)
                if rho_t > 4.0:
                    r = self._rect(rho_t, rho_inf)
                    v_hat = (st["v"] / (1 - b2t)).sqrt_().add_(g["eps"])
                    p.addcdiv_(m_hat, v_hat, value=-g["lr"] * r)
                else:
                    p.add_(m_hat, alpha=-g["lr"])
        return loss


class Lamb(_LrMixin, Optimizer):
    def __init__(self, params, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-6, weight_decay=0.0, clamp_value=None):
        super().__init__(params, dict(lr=lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay,
                                      clamp_value=clamp_value))

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for g in self.param_groups:
            b1, b2 = g["beta1"], g["beta2"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["t"], st["m"], st["v"] = 0, torch.zeros_like(p), torch.zeros_like(p)
                st["t"] += 1
                t = st["t"]
                st["m"].mul_(b1).add_(p.grad, alpha=1 - b1)
                st["v"].mul_(b2).addcmul_(p.grad, p.grad, value=1 - b2)
                u = (st["m"] / (1 - b1 ** t)) / ((st["v"] / (1 - b2 ** t)).sqrt_().add_(g["eps"]))
                if g["weight_decay"]:
                    u.add_(p, alpha=g["weight_decay"])
                pn, un = p.norm(), u.norm()
                trust = torch.where((pn > 0) & (un > 0), pn / un, torch.ones_like(pn))
                if g["clamp_value"] is not None:
                    trust = trust.clamp(max=g["clamp_value"])
                p.sub_(g["lr"] * trust * u)
                st["last_trust"] = float(trust)
        return loss


class Lars(_LrMixin, Optimizer):
    def __init__(self, params, lr=0.1, momentum=0.9, weight_decay=1e-4, trust_coefficient=0.001, clip=False,
                 eps=1e-8):
        super().__init__(params, dict(lr=lr, momentum=momentum, weight_decay=weight_decay,
                                      trust_coefficient=trust_coefficient, clip=clip, eps=eps))

    @classmethod
    def larc(cls, params, lr=0.1, **kw):
        return cls(params, lr=lr, clip=True, **kw)

    @staticmethod
    def local_lr(lr, trust, wd, eps, clip, w_norm, g_norm):
        denom = g_norm + wd * w_norm + eps
        if denom < eps:
            return lr
        local = trust * w_norm / denom
        return min(local, lr) if clip else local

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["v"] = torch.zeros_like(p)
                llr = self.local_lr(g["lr"], g["trust_coefficient"], g["weight_decay"], g["eps"], g["clip"],
                                    float(p.norm()), float(p.grad.norm()))
                eff = p.grad + g["weight_decay"] * p if g["weight_decay"] > 0 else p.grad
                st["v"].mul_(g["momentum"]).add_(eff, alpha=llr)
                p.sub_(st["v"])
        return loss


class Adafactor(_LrMixin, Optimizer):
    def __init__(self, params, lr=None, decay_factor=0.8, min_dim_size_to_factor=128, clipping_threshold=1.0,
                 min_learning_rate=1e-6, warmup_init=False):
        super().__init__(params, dict(lr=lr, decay_factor=decay_factor, min_dim=min_dim_size_to_factor,
                                      clip=clipping_threshold, min_lr=min_learning_rate, warmup_init=warmup_init))
        self.t = 0

    def relative_step_size(self) -> float:
        g = self.param_groups[0]
        t = max(float(self.t), 1.0)
        step = min(1e-6, 1.0 / math.sqrt(t)) if g["warmup_init"] else 1.0 / math.sqrt(t)
        return max(step, g["min_lr"])

    def get_learning_rate(self) -> float:
        lr = self.param_groups[0]["lr"]
        return lr if lr is not None else self.relative_step_size()

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self.t += 1
        for g in self.param_groups:
            lr = g["lr"] if g["lr"] is not None else self.relative_step_size()
            b2 = 1.0 - self.t ** (-g["decay_factor"])
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float()
                if g["clip"] is not None:
                    rms = grad.square().mean().sqrt()
                    if rms > g["clip"]:
                        grad = grad * (g["clip"] / rms)
                rows = p.shape[0] if p.dim() >= 2 else p.numel()
                g2 = grad.reshape(rows, -1).square()
                cols = g2.shape[1]
                st = self.state[p]
                factored = p.dim() >= 2 and min(rows, cols) >= g["min_dim"]
                if not st:
                    if factored:
                        st["row"] = torch.zeros(rows, device=p.device)
                        st["col"] = torch.zeros(cols, device=p.device)
                    else:
                        st["v"] = torch.zeros(rows, cols, device=p.device)
                    if g["lr"] is not None:
                        st["m"] = torch.zeros(rows, cols, device=p.device)
                if factored:
                    st["row"].mul_(b2).add_(g2.mean(1), alpha=1 - b2)
                    st["col"].mul_(b2).add_(g2.mean(0), alpha=1 - b2)
                    rm = st["row"].mean()
                    v = st["row"][:, None] * st["col"][None, :] / torch.where(rm > 0, rm, torch.ones_like(rm))
                else:
                    st["v"].mul_(b2).add_(g2, alpha=1 - b2)
                    v = st["v"]
                upd = grad.reshape(rows, cols) / v.sqrt().clamp_min(1e-30)
                if "m" in st:
                    st["m"].mul_(0.9).add_(upd, alpha=0.1)
                    upd = st["m"]
                p.sub_((lr * upd).reshape(p.shape).to(p.dtype))
        return loss


class Sophia(_LrMixin, Optimizer):
    def __init__(self, params, lr=1e-4, beta1=0.965, beta2=0.99, rho=0.04, weight_decay=0.1, hessian_period=10,
                 eps=1e-8):
        super().__init__(params, dict(lr=lr, beta1=beta1, beta2=beta2, rho=rho, weight_decay=weight_decay,
                                      eps=eps))
        self.hessian_period = hessian_period
        self.t = 0

    def should_update_hessian(self) -> bool:
        return self.t % self.hessian_period == 0

    @torch.no_grad()
    def update_hessian(self, generator: torch.Generator | None = None):
        """Hutchinson update from the current gradients with a fresh
        Rademacher vector z per tensor: h <- b2*h + (1-b2)*(g*z)^2."""
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self._state(p)
                z = torch.randint(0, 2, p.shape, device=p.device, generator=generator).to(p.dtype).mul_(2).sub_(1)
                st["h"].mul_(g["beta2"]).add_((p.grad * z).square(), alpha=1 - g["beta2"])

    def _state(self, p):
        st = self.state[p]
        if not st:
            st["m"], st["h"] = torch.zeros_like(p), torch.zeros_like(p)
        return st

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self.t += 1
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self._state(p)
                st["m"].mul_(g["beta1"]).add_(p.grad, alpha=1 - g["beta1"])
                d = (g["rho"] * st["h"]).clamp_min(g["eps"])
                upd = (st["m"] / d).clamp_(-1, 1).mul_(d)
                if g["weight_decay"]:
                    upd.add_(p, alpha=g["weight_decay"])
                p.sub_(upd, alpha=g["lr"])
        return loss
