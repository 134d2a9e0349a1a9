"""Learning-rate range test.

The learning rate rises from `min_lr` to `max_lr` over `num_iterations`
steps (exponential: min * (max/min)^(i/n); linear); each step's loss is
smoothed by a bias-corrected EMA (Adam-style: EMA from 0, divided by
1 - beta^(i+1)); the run stops when the smoothed loss exceeds
`divergence_threshold` times the best one. Suggestions: the LR at the most
negative d(smoothed loss)/d(log lr), or best-loss LR / 10 (conservative).

`bias_correction="reference"` reproduces lr_finder.rs:284-296 exactly: the
EMA is seeded with the first loss and still divided by 1 - beta^(i+1), which
inflates the first smoothed losses (x50 at beta 0.98) and makes the
steepest-descent suggestion land on the first steps.

Reference parity: scirs2-neural/src/training/lr_finder.rs:61-600
(LRScheduleType, LRFinderConfig, LRFinderResult.from_losses, LRFinder
next_lr / record_loss, find_optimal_lr).
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field


class LRScheduleType(enum.Enum):
    EXPONENTIAL = "exponential"
    LINEAR = "linear"


class LRFinderStatus(enum.Enum):
    CONTINUE = "continue"
    COMPLETE = "complete"
    DIVERGED = "diverged"


@dataclass
class LRFinderConfig:
    min_lr: float = 1e-7
    max_lr: float = 10.0
    num_iterations: int = 100
    schedule: LRScheduleType = LRScheduleType.EXPONENTIAL
    smoothing_factor: float = 0.98
    divergence_threshold: float = 5.0
    accumulation_steps: int = 1
    bias_correction: str = "standard"  # "standard" | "reference"

    def validate(self):
        if self.min_lr <= 0:
            raise ValueError("min_lr must be positive")
        if self.max_lr <= self.min_lr:
            raise ValueError("max_lr must be greater than min_lr")
        if self.num_iterations <= 0:
            raise ValueError("num_iterations must be positive")
        if not 0.0 <= self.smoothing_factor < 1.0:
            raise ValueError("smoothing_factor must be in [0, 1)")
        if self.divergence_threshold <= 1.0:
            raise ValueError("divergence_threshold must be > 1")
        return self

    def lr_at_step(self, step: int) -> float:
        t = step / max(self.num_iterations, 1)
        if self.schedule == LRScheduleType.EXPONENTIAL:
            return self.min_lr * (self.max_lr / self.min_lr) ** t
        return self.min_lr + (self.max_lr - self.min_lr) * t


@dataclass
class LRFinderPoint:
    step: int
    lr: float
    raw_loss: float
    smoothed_loss: float
    loss_gradient: float | None = None


def _smooth(beta: float, i: int, prev: float, loss: float, mode: str = "standard") -> tuple[float, float]:
    if mode == "reference":
        ema = loss if i == 0 else beta * prev + (1.0 - beta) * loss
    else:
        ema = beta * (prev if i else 0.0) + (1.0 - beta) * loss
    corr = 1.0 - beta ** (i + 1)
    return ema, (ema / corr if abs(corr) > 1e-15 else loss)


@dataclass
class LRFinderResult:
    points: list = field(default_factory=list)
    diverged: bool = False
    divergence_step: int | None = None
    best_loss: float = math.inf
    best_loss_lr: float = 0.0

    @classmethod
    def from_losses(cls, losses, config: LRFinderConfig) -> "LRFinderResult":
        r = cls(best_loss_lr=config.min_lr)
        ema = 0.0
        for i, raw in enumerate(losses):
            lr = config.lr_at_step(i)
            ema, sm = _smooth(config.smoothing_factor, i, ema, raw, config.bias_correction)
            if sm < r.best_loss:
                r.best_loss, r.best_loss_lr = sm, lr
            r.points.append(LRFinderPoint(i, lr, raw, sm))
            if r.best_loss > 0 and sm > r.best_loss * config.divergence_threshold:
                r.diverged, r.divergence_step = True, i
                break
        for a, b in zip(r.points[:-1], r.points[1:]):
            d = math.log(b.lr) - math.log(a.lr)
            if abs(d) > 1e-300:
                b.loss_gradient = (b.smoothed_loss - a.smoothed_loss) / d
        return r

    def suggested_lr(self) -> float | None:
        g = [(p.loss_gradient, p.lr) for p in self.points if p.loss_gradient is not None]
        return min(g)[1] if g else None

    def suggested_lr_conservative(self) -> float:
        return self.best_loss_lr / 10.0

    def learning_rates(self):
        return [p.lr for p in self.points]

    def raw_losses(self):
        return [p.raw_loss for p in self.points]

    def smoothed_losses(self):
        return [p.smoothed_loss for p in self.points]

    def summary(self) -> str:
        s = self.suggested_lr()
        return (f"LR range test: {len(self.points)} points, best loss {self.best_loss:.4g} at lr "
                f"{self.best_loss_lr:.3g}, suggested lr {s if s is None else f'{s:.3g}'}"
                + (f", diverged at step {self.divergence_step}" if self.diverged else ""))


class LRFinder:
    def __init__(self, config: LRFinderConfig | None = None):
        self.config = (config or LRFinderConfig()).validate()
        self.reset()

    def reset(self):
        self.step, self.ema, self.best = 0, 0.0, math.inf
        self.raw: list[float] = []
        self.finished = self.diverged = False

    def next_lr(self) -> float | None:
        return None if self.finished else self.config.lr_at_step(self.step)

    def record_loss(self, loss: float) -> LRFinderStatus:
        if self.finished:
            return LRFinderStatus.DIVERGED if self.diverged else LRFinderStatus.COMPLETE
        self.raw.append(float(loss))
        self.ema, sm = _smooth(self.config.smoothing_factor, self.step, self.ema, float(loss),
                               self.config.bias_correction)
        self.best = min(self.best, sm)
        if self.best > 0 and sm > self.best * self.config.divergence_threshold:
            self.finished = self.diverged = True
            return LRFinderStatus.DIVERGED
        self.step += 1
        if self.step >= self.config.num_iterations:
            self.finished = True
            return LRFinderStatus.COMPLETE
        return LRFinderStatus.CONTINUE

    def result(self) -> LRFinderResult:
        return LRFinderResult.from_losses(self.raw, self.config)


def find_optimal_lr(train_step, set_lr, config: LRFinderConfig | None = None, state=None, restore=None):
    """Run the range test: `set_lr(lr)`, `loss = train_step()` until done.
    `state()` / `restore(s)` (optional) save and put back the model so the
    test leaves it unchanged."""
    saved = state() if state is not None else None
    f = LRFinder(config)
    while (lr := f.next_lr()) is not None:
        set_lr(lr)
        if f.record_loss(float(train_step())) != LRFinderStatus.CONTINUE:
            break
    if restore is not None:
        restore(saved)
    return f.result()
