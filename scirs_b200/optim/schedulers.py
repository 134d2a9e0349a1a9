"""Learning-rate schedules (scirs2-neural/src/training/schedulers.rs:71-800).

Each schedule is a pure function of the epoch / step (`get_lr(epoch)`, as
in the reference's LRScheduler trait). `Scheduled(optimizer, schedule)`
drives any optimizer of this framework (or torch.optim) from it.
"""
from __future__ import annotations

import math


class LRScheduler:
    def get_lr(self, epoch: int) -> float:
        raise NotImplementedError

    def get_lr_at_step(self, step: int, epoch: int) -> float:
        return self.get_lr(epoch)

    def name(self) -> str:
        return type(self).__name__


class ConstantLR(LRScheduler):
    def __init__(self, lr):
        self.lr = lr

    def get_lr(self, epoch):
        return self.lr


class StepLR(LRScheduler):
    def __init__(self, base_lr, step_size, gamma=0.1):
        self.base_lr, self.step_size, self.gamma = base_lr, max(1, step_size), gamma

    def get_lr(self, epoch):
        return self.base_lr * self.gamma ** (epoch // self.step_size)


class MultiStepLR(LRScheduler):
    def __init__(self, base_lr, milestones, gamma=0.1):
        self.base_lr, self.milestones, self.gamma = base_lr, sorted(milestones), gamma

    def get_lr(self, epoch):
        return self.base_lr * self.gamma ** sum(1 for m in self.milestones if epoch >= m)


class ExponentialLR(LRScheduler):
    def __init__(self, base_lr, gamma):
        self.base_lr, self.gamma = base_lr, gamma

    def get_lr(self, epoch):
        return self.base_lr * self.gamma**epoch


class CosineAnnealingLR(LRScheduler):
    def __init__(self, base_lr, t_max, eta_min=0.0):
        self.base_lr, self.t_max, self.eta_min = base_lr, max(1, t_max), eta_min

    def get_lr(self, epoch):
        e = min(epoch, self.t_max)
        return self.eta_min + (self.base_lr - self.eta_min) * 0.5 * (1 + math.cos(math.pi * e / self.t_max))


class CosineAnnealingWarmRestarts(LRScheduler):
    def __init__(self, base_lr, t_0, t_mult=1, eta_min=0.0):
        self.base_lr, self.t_0, self.t_mult, self.eta_min = base_lr, max(1, t_0), max(1, t_mult), eta_min

    def get_lr(self, epoch):
        t_i, t_cur = self.t_0, epoch
        while t_cur >= t_i:
            t_cur -= t_i
            t_i *= self.t_mult
        return self.eta_min + (self.base_lr - self.eta_min) * 0.5 * (1 + math.cos(math.pi * t_cur / t_i))


class LinearWarmup(LRScheduler):
    def __init__(self, base_lr, warmup_steps, start_lr=0.0):
        self.base_lr, self.warmup, self.start = base_lr, max(1, warmup_steps), start_lr

    def get_lr(self, epoch):
        if epoch >= self.warmup:
            return self.base_lr
        return self.start + (self.base_lr - self.start) * epoch / self.warmup


class WarmupCosine(LRScheduler):
    """Linear warmup to base_lr, then cosine decay to min_lr at total_steps."""

    def __init__(self, base_lr, warmup_steps, total_steps, min_lr=0.0):
        self.base_lr, self.warmup, self.total, self.min_lr = base_lr, warmup_steps, max(1, total_steps), min_lr

    def get_lr(self, epoch):
        if epoch < self.warmup:
            return self.base_lr * (epoch + 1) / self.warmup
        p = min(1.0, (epoch - self.warmup) / max(1, self.total - self.warmup))
        return self.min_lr + (self.base_lr - self.min_lr) * 0.5 * (1 + math.cos(math.pi * p))


class OneCycleLR(LRScheduler):
    def __init__(self, max_lr, total_steps, pct_start=0.3, div_factor=25.0, final_div_factor=1e4):
        self.max_lr, self.total = max_lr, max(1, total_steps)
        self.pct_start = min(max(pct_start, 0.0), 1.0)
        self.div = div_factor if div_factor > 0 else 25.0
        self.fdiv = final_div_factor if final_div_factor > 0 else 1e4

    def get_lr(self, step):
        pct = min(step, self.total) / self.total
        lo = self.max_lr / self.div
        fin = lo / self.fdiv
        if pct <= self.pct_start:
            ph = pct / self.pct_start if self.pct_start > 0 else 1.0
            return lo + (self.max_lr - lo) * 0.5 * (1 - math.cos(math.pi * ph))
        rem = 1.0 - self.pct_start
        ph = (pct - self.pct_start) / rem if rem > 0 else 1.0
        return fin + (self.max_lr - fin) * 0.5 * (1 + math.cos(math.pi * ph))

    def get_lr_at_step(self, step, epoch):
        return self.get_lr(step)


class PolynomialLR(LRScheduler):
    def __init__(self, base_lr, total_steps, power=1.0, end_lr=0.0):
        self.base_lr, self.total, self.power, self.end_lr = base_lr, max(1, total_steps), power, end_lr

    def get_lr(self, epoch):
        p = min(epoch, self.total) / self.total
        return (self.base_lr - self.end_lr) * (1 - p) ** self.power + self.end_lr


class ReduceOnPlateau(LRScheduler):
    """Multiply the lr by `factor` when the monitored metric has not improved
    for `patience` epochs (call `observe(metric)` once per epoch)."""

    def __init__(self, base_lr, factor=0.1, patience=10, min_lr=0.0, threshold=1e-4, mode="min"):
        self.lr, self.factor, self.patience, self.min_lr = base_lr, factor, patience, min_lr
        self.threshold, self.mode = threshold, mode
        self.best, self.bad = None, 0

    def observe(self, metric: float) -> float:
        better = self.best is None or (
            metric < self.best - self.threshold if self.mode == "min" else metric > self.best + self.threshold
        )
        if better:
            self.best, self.bad = metric, 0
        else:
            self.bad += 1
            if self.bad > self.patience:
                self.lr = max(self.min_lr, self.lr * self.factor)
                self.bad = 0
        return self.lr

    def get_lr(self, epoch):
        return self.lr


class CyclicLR(LRScheduler):
    def __init__(self, base_lr, max_lr, step_size_up=2000, mode="triangular", gamma=1.0):
        self.base_lr, self.max_lr, self.step, self.mode, self.gamma = base_lr, max_lr, max(1, step_size_up), mode, gamma

    def get_lr(self, it):
        cycle = math.floor(1 + it / (2 * self.step))
        x = abs(it / self.step - 2 * cycle + 1)
        amp = (self.max_lr - self.base_lr) * max(0.0, 1 - x)
        if self.mode == "triangular2":
            amp /= 2 ** (cycle - 1)
        elif self.mode == "exp_range":
            amp *= self.gamma**it
        return self.base_lr + amp


class ChainedScheduler(LRScheduler):
    """Product of two schedules normalised by the second's base value."""

    def __init__(self, a: LRScheduler, b: LRScheduler):
        self.a, self.b = a, b

    def get_lr(self, epoch):
        b0 = self.b.get_lr(0) or 1.0
        return self.a.get_lr(epoch) * self.b.get_lr(epoch) / b0


def set_lr(optimizer, lr: float):
    if hasattr(optimizer, "set_learning_rate"):
        optimizer.set_learning_rate(lr)
    elif hasattr(optimizer, "lr") and not hasattr(optimizer, "param_groups"):
        optimizer.lr = lr
    else:
        for g in optimizer.param_groups:
            g["lr"] = lr
    if hasattr(optimizer, "lr"):
        optimizer.lr = lr


class Scheduled:
    """Binds a schedule to an optimizer: call `step()` after every optimizer step."""

    def __init__(self, optimizer, schedule: LRScheduler):
        self.opt, self.schedule, self.n = optimizer, schedule, 0
        set_lr(optimizer, schedule.get_lr_at_step(0, 0))

    def step(self, epoch: int | None = None):
        self.n += 1
        lr = self.schedule.get_lr_at_step(self.n, self.n if epoch is None else epoch)
        set_lr(self.opt, lr)
        return lr
