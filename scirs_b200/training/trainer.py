"""EnhancedTrainer: a configurable training loop for torch modules with
learning-rate warm-up, gradient accumulation, gradient clipping, periodic
validation, early stopping, checkpoint callbacks, progress logging and an
optional per-layer profiler; and the TrainingProfiler it uses.

Reference parity: scirs2-neural/src/training/enhanced_trainer.rs:40-1590
(EnhancedTrainingConfig, ValidationConfig, EarlyStoppingConfig,
LRWarmupConfig / WarmupSchedule, GradientAccumulationSettings,
ProgressConfig, ProfilingConfig, TrainingState, OperationTiming /
ProfilingResults) and training/profiler.rs:45-1368 (LayerProfile,
BatchStats, EpochStats, ProfilePhase, Bottleneck, TrainingProfiler).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from .metrics_tracker import MetricGoal, MetricsTracker


@dataclass
class LRWarmupConfig:
    warmup_steps: int = 0
    schedule: str = "linear"  # linear | cosine | exponential
    start_factor: float = 0.0

    def factor(self, step: int) -> float:
        if self.warmup_steps <= 0 or step >= self.warmup_steps:
            return 1.0
        t = step / self.warmup_steps
        if self.schedule == "cosine":
            f = 0.5 * (1 - math.cos(math.pi * t))
        elif self.schedule == "exponential":
            f = t ** 2
        else:
            f = t
        return self.start_factor + (1 - self.start_factor) * f


@dataclass
class EarlyStoppingConfig:
    enabled: bool = False
    monitor: str = "val_loss"
    patience: int = 5
    min_delta: float = 0.0
    goal: MetricGoal = MetricGoal.MINIMIZE
    restore_best: bool = True


@dataclass
class EnhancedTrainingConfig:
    epochs: int = 10
    grad_accumulation: int = 1
    max_grad_norm: float = 0.0
    validation_every: int = 1
    log_every: int = 50
    warmup: LRWarmupConfig = field(default_factory=LRWarmupConfig)
    early_stopping: EarlyStoppingConfig = field(default_factory=EarlyStoppingConfig)
    profile: bool = False


@dataclass
class TrainingState:
    epoch: int = 0
    global_step: int = 0
    best_value: float | None = None
    best_epoch: int = -1
    stop: bool = False
    history: dict = field(default_factory=dict)


@dataclass
class LayerProfile:
    name: str
    forward_s: list = field(default_factory=list)
    backward_s: list = field(default_factory=list)

    def avg_forward(self) -> float:
        return sum(self.forward_s) / len(self.forward_s) if self.forward_s else 0.0

    def avg_backward(self) -> float:
        return sum(self.backward_s) / len(self.backward_s) if self.backward_s else 0.0

    def total_time(self) -> float:
        return sum(self.forward_s) + sum(self.backward_s)


@dataclass
class Bottleneck:
    layer: str
    share: float
    phase: str


class TrainingProfiler:
    """Per-layer forward / backward wall time through module hooks (device
    work is synchronised around each measured layer when on CUDA, so use it
    for diagnosis, not for throughput numbers)."""

    def __init__(self, model: nn.Module | None = None, enabled: bool = True):
        self.enabled = enabled
        self.layers: dict[str, LayerProfile] = {}
        self.phase_times: dict[str, float] = {}
        self._hooks = []
        if model is not None and enabled:
            self.attach(model)

    def _sync(self, t):
        if isinstance(t, torch.Tensor) and t.is_cuda:
            torch.cuda.synchronize(t.device)

    def attach(self, model: nn.Module):
        for name, mod in model.named_modules():
            if not name or list(mod.children()):
                continue
            prof = self.layers.setdefault(name, LayerProfile(name))
            start = {}

            def fpre(m, inp, _s=start):
                self._sync(inp[0] if inp else None)
                _s["f"] = time.perf_counter()

            def fpost(m, inp, out, _p=prof, _s=start):
                self._sync(out)
                _p.forward_s.append(time.perf_counter() - _s["f"])

            def bpre(m, gout, _s=start):
                self._sync(gout[0] if gout else None)
                _s["b"] = time.perf_counter()

            def bpost(m, gin, gout, _p=prof, _s=start):
                self._sync(gin[0] if gin and gin[0] is not None else None)
                if "b" in _s:
                    _p.backward_s.append(time.perf_counter() - _s["b"])

            self._hooks += [mod.register_forward_pre_hook(fpre), mod.register_forward_hook(fpost),
                            mod.register_full_backward_pre_hook(bpre), mod.register_full_backward_hook(bpost)]

    def phase(self, name: str, seconds: float):
        self.phase_times[name] = self.phase_times.get(name, 0.0) + seconds

    def bottlenecks(self, top: int = 3) -> list[Bottleneck]:
        total = sum(p.total_time() for p in self.layers.values()) or 1.0
        out = []
        for p in self.layers.values():
            f, b = sum(p.forward_s), sum(p.backward_s)
            out.append(Bottleneck(p.name, (f + b) / total, "forward" if f >= b else "backward"))
        return sorted(out, key=lambda x: -x.share)[:top]

    def detach(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []


class EnhancedTrainer:
    def __init__(self, model: nn.Module, optimizer, loss_fn, config: EnhancedTrainingConfig | None = None,
                 callbacks=None, log=print):
        self.model, self.opt, self.loss_fn = model, optimizer, loss_fn
        self.cfg = config or EnhancedTrainingConfig()
        self.callbacks = list(callbacks or [])
        self.log = log
        self.state = TrainingState()
        self.tracker = MetricsTracker()
        self.tracker.register_metric("loss", MetricGoal.MINIMIZE)
        self.profiler = TrainingProfiler(model) if self.cfg.profile else None
        self._base_lrs = [g["lr"] for g in optimizer.param_groups]
        self._best_state = None

    def _set_warmup_lr(self):
        f = self.cfg.warmup.factor(self.state.global_step)
        for g, lr in zip(self.opt.param_groups, self._base_lrs):
            g["lr"] = lr * f

    def evaluate(self, data) -> float:
        self.model.eval()
        tot, n = 0.0, 0
        with torch.no_grad():
            for x, y in data:
                tot += float(self.loss_fn(self.model(x), y)) * len(x)
                n += len(x)
        self.model.train()
        return tot / max(n, 1)

    def fit(self, train_data, val_data=None) -> TrainingState:
        cfg, st = self.cfg, self.state
        es = cfg.early_stopping
        self.tracker.register_metric(es.monitor, es.goal)
        for epoch in range(cfg.epochs):
            st.epoch = epoch
            self.model.train()
            t0 = time.perf_counter()
            self.opt.zero_grad(set_to_none=True)
            for i, (x, y) in enumerate(train_data):
                loss = self.loss_fn(self.model(x), y) / cfg.grad_accumulation
                loss.backward()
                self.tracker.record_batch("loss", float(loss) * cfg.grad_accumulation)
                if (i + 1) % cfg.grad_accumulation == 0:
                    if cfg.max_grad_norm > 0:
                        torch.nn.utils.clip_grad_norm_(self.model.parameters(), cfg.max_grad_norm)
                    self._set_warmup_lr()
                    self.opt.step()
                    self.opt.zero_grad(set_to_none=True)
                    st.global_step += 1
                    if cfg.log_every and st.global_step % cfg.log_every == 0:
                        self.log(f"epoch {epoch} step {st.global_step} loss {float(loss) * cfg.grad_accumulation:.4f}")
            self.tracker.end_epoch("loss", epoch)
            if self.profiler is not None:
                self.profiler.phase("train", time.perf_counter() - t0)
            logs = {"loss": self.tracker.metrics["loss"].epoch_values[-1][1]}
            if val_data is not None and (epoch + 1) % cfg.validation_every == 0:
                logs["val_loss"] = self.evaluate(val_data)
            for k, v in logs.items():
                st.history.setdefault(k, []).append(v)
            if es.enabled and es.monitor in logs:
                v = logs[es.monitor]
                better = st.best_value is None or (
                    v < st.best_value - es.min_delta if es.goal == MetricGoal.MINIMIZE else v > st.best_value + es.min_delta)
                if better:
                    st.best_value, st.best_epoch = v, epoch
                    if es.restore_best:
                        self._best_state = {k: t.detach().clone() for k, t in self.model.state_dict().items()}
                elif epoch - st.best_epoch >= es.patience:
                    st.stop = True
            for cb in self.callbacks:
                if hasattr(cb, "on_epoch_end") and cb.on_epoch_end(epoch, logs) is True:
                    st.stop = True
            if st.stop:
                break
        if es.enabled and es.restore_best and self._best_state is not None:
            self.model.load_state_dict(self._best_state)
        return st
