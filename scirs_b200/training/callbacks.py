"""More training callbacks: timing-keyed dispatch, function callbacks,
gradient clipping, learning-rate schedules driven by epochs / batches /
plateaus, and a visualization callback.

They follow the `training.history.Callback` interface
(on_train_begin / on_epoch_begin / on_batch_end / on_epoch_end /
on_train_end, plus `on_before_step(model)`, which `Sequential.fit` calls
between the backward and the optimizer step). Learning-rate callbacks set the
`lr` of every parameter group of `model.optimizer`.

Reference parity: scirs2-neural/src/callbacks/mod.rs:14-90 (CallbackTiming,
FunctionCallback), callback_manager.rs:16-120, gradient_clipping.rs:14-140,
learning_rate_scheduler.rs:12-330 (StepDecay, ReduceOnPlateau,
CosineAnnealingLR, ScheduleMethod), visualization_callback.rs:13-160.
"""
from __future__ import annotations

import math
import os
from enum import Enum

import torch

from .history import Callback


class CallbackTiming(Enum):
    BEFORE_TRAINING = "before_training"
    BEFORE_EPOCH = "before_epoch"
    BEFORE_BATCH = "before_batch"
    AFTER_BATCH = "after_batch"
    AFTER_EPOCH = "after_epoch"
    AFTER_TRAINING = "after_training"


class FunctionCallback(Callback):
    """Runs fn(context) at one timing; context = {"epoch", "batch", "model", "logs"}."""

    def __init__(self, timing: CallbackTiming, fn):
        self.timing, self.fn = timing, fn
        self.stop_training = False

    def _run(self, t, **ctx):
        if t is self.timing and self.fn(ctx) is True:
            self.stop_training = True

    def on_train_begin(self, model, logs=None):
        self._run(CallbackTiming.BEFORE_TRAINING, model=model, logs=logs)

    def on_epoch_begin(self, epoch, model, logs=None):
        self._run(CallbackTiming.BEFORE_EPOCH, epoch=epoch, model=model, logs=logs)

    def on_batch_end(self, step, model, logs=None):
        self._run(CallbackTiming.AFTER_BATCH, batch=step, model=model, logs=logs)

    def on_epoch_end(self, epoch, model, logs=None):
        self._run(CallbackTiming.AFTER_EPOCH, epoch=epoch, model=model, logs=logs)

    def on_train_end(self, model, logs=None):
        self._run(CallbackTiming.AFTER_TRAINING, model=model, logs=logs)


class CallbackManager(Callback):
    """A list of callbacks behind one callback: dispatches every event to all of them in order and
    stops training when any asks to."""

    def __init__(self, callbacks=None):
        self.callbacks = list(callbacks or [])

    def add(self, cb):
        self.callbacks.append(cb)
        return self

    @property
    def stop_training(self):
        return any(getattr(c, "stop_training", False) for c in self.callbacks)

    def on_train_begin(self, model, logs=None):
        for c in self.callbacks:
            c.on_train_begin(model, logs)

    def on_epoch_begin(self, epoch, model, logs=None):
        for c in self.callbacks:
            c.on_epoch_begin(epoch, model, logs)

    def on_batch_end(self, step, model, logs=None):
        for c in self.callbacks:
            c.on_batch_end(step, model, logs)

    def on_before_step(self, model):
        for c in self.callbacks:
            if hasattr(c, "on_before_step"):
                c.on_before_step(model)

    def on_epoch_end(self, epoch, model, logs=None):
        for c in self.callbacks:
            c.on_epoch_end(epoch, model, logs)

    def on_train_end(self, model, logs=None):
        for c in self.callbacks:
            c.on_train_end(model, logs)


class GradientClipping(Callback):
    """Clips the model's gradients before every optimizer step, by global norm or by value; records
    whether clipping happened and the scale applied (global norm)."""

    def __init__(self, max_norm: float, method: str = "global_norm", log_stats: bool = False):
        if method not in ("global_norm", "value"):
            raise ValueError("method must be 'global_norm' or 'value'")
        self.max_norm, self.method, self.log_stats = float(max_norm), method, log_stats
        self.clipping_applied, self.clipping_ratio = False, None
        self.stop_training = False

    @staticmethod
    def by_global_norm(max_norm, log_stats=False):
        return GradientClipping(max_norm, "global_norm", log_stats)

    @staticmethod
    def by_value(max_value, log_stats=False):
        return GradientClipping(max_value, "value", log_stats)

    @torch.no_grad()
    def on_before_step(self, model):
        grads = [p.grad for p in model.parameters() if p.grad is not None]
        if not grads:
            return
        if self.method == "value":
            self.clipping_applied = any(bool((g.abs() > self.max_norm).any()) for g in grads)
            for g in grads:
                g.clamp_(-self.max_norm, self.max_norm)
            self.clipping_ratio = None
        else:
            total = torch.linalg.vector_norm(torch.stack([torch.linalg.vector_norm(g.float()) for g in grads]))
            self.clipping_applied = bool(total > self.max_norm)
            self.clipping_ratio = float(self.max_norm / total) if self.clipping_applied else 1.0
            if self.clipping_applied:
                for g in grads:
                    g.mul_(self.clipping_ratio)
        if self.log_stats and self.clipping_applied:
            print(f"gradient clipping applied (ratio {self.clipping_ratio})")


def _set_lr(model, lr):
    if getattr(model, "optimizer", None) is None and hasattr(model, "_ensure_opt"):
        model._ensure_opt()
    opt = getattr(model, "optimizer", None)
    if opt is None:
        return
    if hasattr(opt, "set_learning_rate"):  # the framework's optimizers
        opt.set_learning_rate(lr)
        return
    for g in opt.param_groups:
        g["lr"] = lr


class _LRCallback(Callback):
    def __init__(self, method: str):
        if method not in ("epoch", "batch"):
            raise ValueError("method must be 'epoch' or 'batch'")
        self.method, self.step_count, self.current_lr = method, 0, None
        self.stop_training = False

    def lr_at(self, step: int) -> float:
        raise NotImplementedError

    def _advance(self, model):
        self.current_lr = self.lr_at(self.step_count)
        _set_lr(model, self.current_lr)
        self.step_count += 1

    def on_epoch_begin(self, epoch, model, logs=None):
        if self.method == "epoch":
            self._advance(model)

    def on_before_step(self, model):
        if self.method == "batch":
            self._advance(model)


class StepDecay(_LRCallback):
    """lr = initial * factor ** (step // step_size)."""

    def __init__(self, initial_lr, factor, step_size, method="epoch"):
        super().__init__(method)
        self.initial_lr, self.factor, self.step_size = initial_lr, factor, max(1, int(step_size))

    def lr_at(self, step):
        return self.initial_lr * self.factor ** (step // self.step_size)


class CosineAnnealingLR(_LRCallback):
    """lr = min + (initial - min) (1 + cos(pi * (step mod T) / T)) / 2."""

    def __init__(self, initial_lr, min_lr, t_max, method="epoch"):
        super().__init__(method)
        self.initial_lr, self.min_lr, self.t_max = initial_lr, min_lr, max(1, int(t_max))

    def lr_at(self, step):
        t = step % self.t_max
        return self.min_lr + (self.initial_lr - self.min_lr) * (1 + math.cos(math.pi * t / self.t_max)) / 2


class ReduceOnPlateau(Callback):
    """Multiplies the lr by `factor` (not below min_lr) when the monitored loss has not improved by
    more than `threshold` for `patience` epochs."""

    def __init__(self, initial_lr, factor=0.1, patience=10, threshold=1e-4, min_lr=0.0, monitor="val_loss"):
        self.current_lr, self.factor, self.patience = initial_lr, factor, patience
        self.threshold, self.min_lr, self.monitor = threshold, min_lr, monitor
        self.best, self.counter = None, 0
        self.stop_training = False

    def on_train_begin(self, model, logs=None):
        _set_lr(model, self.current_lr)

    def on_epoch_end(self, epoch, model, logs=None):
        logs = logs or {}
        v = logs.get(self.monitor, logs.get("loss"))
        if v is None:
            return
        if self.best is None or v < self.best - self.threshold:
            self.best, self.counter = v, 0
            return
        self.counter += 1
        if self.counter >= self.patience:
            self.current_lr = max(self.min_lr, self.current_lr * self.factor)
            _set_lr(model, self.current_lr)
            self.counter = 0


class VisualizationCallback(Callback):
    """Tracks epoch metrics and, every `frequency` epochs, renders them as text plots (and writes
    an SVG per metric under `save_path` when given)."""

    def __init__(self, frequency=1, show_plots=False, save_path=None, tracked_metrics=("loss", "val_loss"),
                 width=80, height=20):
        self.frequency, self.show_plots, self.save_path = max(1, int(frequency)), show_plots, save_path
        self.tracked_metrics, self.width, self.height = list(tracked_metrics), width, height
        self.epoch_history: dict[str, list] = {m: [] for m in self.tracked_metrics}
        self.rendered: list[str] = []
        self.stop_training = False

    def on_epoch_end(self, epoch, model, logs=None):
        from ..utils.visualization import ascii_plot, svg_line_plot

        for m in self.tracked_metrics:
            if logs and m in logs:
                self.epoch_history[m].append(float(logs[m]))
        if (epoch + 1) % self.frequency:
            return
        for m, vals in self.epoch_history.items():
            if not vals:
                continue
            txt = ascii_plot(vals, self.width, self.height, title=m)
            self.rendered.append(txt)
            if self.show_plots:
                print(txt)
            if self.save_path:
                os.makedirs(self.save_path, exist_ok=True)
                svg_line_plot({m: vals}, os.path.join(self.save_path, f"{m}.svg"), title=m)
