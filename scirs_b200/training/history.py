"""Training configuration, history and callbacks.

  TrainingConfig / History   scirs2-neural/src/models/trainer.rs:11-77
  Callbacks                  scirs2-neural/src/callbacks/*.rs (early stopping, checkpoint,
                             LR scheduler, TensorBoard-style logger -> JSONL scalars here)
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import dataclass, field


@dataclass
class TrainingConfig:
    epochs: int = 10
    batch_size: int = 32
    learning_rate: float = 0.01
    shuffle: bool = True
    validation_split: float = 0.2
    verbose: int = 1


@dataclass
class History:
    train_loss: list = field(default_factory=list)
    val_loss: list = field(default_factory=list)
    metrics: dict = field(default_factory=dict)

    def log(self, name, value):
        self.metrics.setdefault(name, []).append(value)


class Callback:
    def on_train_begin(self, model, logs=None): ...
    def on_epoch_begin(self, epoch, model, logs=None): ...
    def on_batch_end(self, step, model, logs=None): ...
    def on_epoch_end(self, epoch, model, logs=None): ...
    def on_train_end(self, model, logs=None): ...

    stop_training = False


class EarlyStopping(Callback):
    def __init__(self, monitor="val_loss", patience=5, min_delta=0.0, mode="min", restore_best_weights=False):
        self.monitor, self.patience, self.min_delta, self.mode = monitor, patience, min_delta, mode
        self.restore = restore_best_weights
        self.best, self.wait, self.best_state = None, 0, None
        self.stopped_epoch = None

    def on_epoch_end(self, epoch, model, logs=None):
        v = (logs or {}).get(self.monitor)
        if v is None or (isinstance(v, float) and math.isnan(v)):
            return
        better = self.best is None or (
            v < self.best - self.min_delta if self.mode == "min" else v > self.best + self.min_delta
        )
        if better:
            self.best, self.wait = v, 0
            if self.restore and hasattr(model, "state_dict"):
                self.best_state = {k: t.detach().clone() for k, t in model.state_dict().items()}
        else:
            self.wait += 1
            if self.wait >= self.patience:
                self.stop_training = True
                self.stopped_epoch = epoch
                if self.restore and self.best_state is not None:
                    model.load_state_dict(self.best_state)


class ModelCheckpoint(Callback):
    """Saves a checkpoint directory (see training.checkpoint) every epoch or
    only when the monitored value improves."""

    def __init__(self, directory, monitor="val_loss", save_best_only=False, mode="min"):
        self.dir, self.monitor, self.best_only, self.mode = directory, monitor, save_best_only, mode
        self.best = None

    def on_epoch_end(self, epoch, model, logs=None):
        from .checkpoint import CheckpointMetadata, save_checkpoint

        logs = logs or {}
        v = logs.get(self.monitor, logs.get("loss"))
        if self.best_only and v is not None and self.best is not None:
            if (self.mode == "min" and v >= self.best) or (self.mode == "max" and v <= self.best):
                return
        if v is not None:
            self.best = v if self.best is None else (min(self.best, v) if self.mode == "min" else max(self.best, v))
        path = os.path.join(self.dir, f"epoch_{epoch:04d}")
        meta = CheckpointMetadata(epoch=epoch, step=epoch, loss=float(logs.get("loss", float("nan"))),
                                  val_loss=logs.get("val_loss"))
        save_checkpoint(path, model.state_dict(), meta)


class LRSchedulerCallback(Callback):
    def __init__(self, optimizer_getter, schedule):
        self.get_opt, self.schedule = optimizer_getter, schedule

    def on_epoch_begin(self, epoch, model, logs=None):
        from ..optim.schedulers import set_lr

        set_lr(self.get_opt(model), self.schedule.get_lr(epoch))


class ScalarLogger(Callback):
    """TensorBoard-style scalar log (scirs2-neural/src/callbacks/tensorboard.rs:14-32)
    written as JSON lines under `log_dir/scalars.jsonl`."""

    def __init__(self, log_dir):
        self.log_dir = log_dir
        os.makedirs(log_dir, exist_ok=True)
        self.path = os.path.join(log_dir, "scalars.jsonl")

    def write(self, tag, value, step):
        with open(self.path, "a") as f:
            f.write(json.dumps({"tag": tag, "value": float(value), "step": int(step), "wall": time.time()}) + "\n")

    def on_epoch_end(self, epoch, model, logs=None):
        for k, v in (logs or {}).items():
            if v is not None:
                self.write(k, v, epoch)
