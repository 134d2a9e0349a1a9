"""Training-metric bookkeeping: per-batch values with exponential smoothing,
per-epoch values, best values under a goal (minimise / maximise), summary
statistics and improvement tracking.

Reference parity: scirs2-neural/src/training/metrics_tracker.rs:42-770
(MetricGoal, MetricEntry, BestMetric, MetricHistory, MetricStats,
MetricsTracker register / record_batch / record_epoch / end_epoch).
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field


class MetricGoal(enum.Enum):
    MINIMIZE = "minimize"
    MAXIMIZE = "maximize"


@dataclass
class BestMetric:
    value: float
    epoch: int


@dataclass
class MetricStats:
    count: int
    mean: float
    std: float
    min: float
    max: float


@dataclass
class MetricHistory:
    goal: MetricGoal
    smoothing: float
    batch_values: list = field(default_factory=list)
    smoothed: list = field(default_factory=list)
    epoch_values: list = field(default_factory=list)
    best: BestMetric | None = None
    _epoch_batches: list = field(default_factory=list)


class MetricsTracker:
    def __init__(self, smoothing: float = 0.0):
        self.default_smoothing = smoothing
        self.metrics: dict[str, MetricHistory] = {}

    def register_metric(self, name: str, goal: MetricGoal = MetricGoal.MINIMIZE, smoothing: float | None = None):
        self.metrics[name] = MetricHistory(goal, self.default_smoothing if smoothing is None else smoothing)

    def _h(self, name) -> MetricHistory:
        if name not in self.metrics:
            self.register_metric(name)
        return self.metrics[name]

    def record_batch(self, name: str, value: float) -> float:
        h = self._h(name)
        v = float(value)
        h.batch_values.append(v)
        h._epoch_batches.append(v)
        prev = h.smoothed[-1] if h.smoothed else v
        s = h.smoothing * prev + (1 - h.smoothing) * v
        h.smoothed.append(s)
        return s

    def _better(self, h: MetricHistory, v: float) -> bool:
        if h.best is None:
            return True
        return v < h.best.value if h.goal == MetricGoal.MINIMIZE else v > h.best.value

    def record_epoch(self, name: str, epoch: int, value: float) -> float | None:
        """Returns the improvement over the previous best (None if not better)."""
        h = self._h(name)
        v = float(value)
        h.epoch_values.append((epoch, v))
        if self._better(h, v):
            imp = None if h.best is None else abs(v - h.best.value)
            h.best = BestMetric(v, epoch)
            return imp if imp is not None else 0.0
        return None

    def end_epoch(self, name: str, epoch: int) -> float | None:
        """Record the mean of the batches seen since the last end_epoch."""
        h = self._h(name)
        if not h._epoch_batches:
            return None
        v = sum(h._epoch_batches) / len(h._epoch_batches)
        h._epoch_batches = []
        return self.record_epoch(name, epoch, v)

    def best(self, name: str) -> BestMetric | None:
        return self.metrics[name].best

    def epochs_since_improvement(self, name: str) -> int:
        h = self.metrics[name]
        if h.best is None or not h.epoch_values:
            return 0
        return h.epoch_values[-1][0] - h.best.epoch

    def stats(self, name: str) -> MetricStats:
        vals = [v for _, v in self.metrics[name].epoch_values] or self.metrics[name].batch_values
        n = len(vals)
        mean = sum(vals) / n
        std = math.sqrt(sum((x - mean) ** 2 for x in vals) / n)
        return MetricStats(n, mean, std, min(vals), max(vals))

    def summary(self) -> dict:
        return {k: {"best": None if h.best is None else h.best.value,
                    "best_epoch": None if h.best is None else h.best.epoch,
                    "last": h.epoch_values[-1][1] if h.epoch_values else (h.batch_values or [None])[-1]}
                for k, h in self.metrics.items()}
