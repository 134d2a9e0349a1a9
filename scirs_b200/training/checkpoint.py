"""Training checkpoints: the reference's directory layout
(scirs2-neural/src/training/checkpoint.rs:380-1060)

    <dir>/model.safetensors            weights (+ metadata architecture/version/epoch/checkpoint)
    <dir>/checkpoint_meta.json         CheckpointMetadata (serde-pretty JSON)
    <dir>/optimizer_state.safetensors  optimizer moments (optional)

plus list / latest / best helpers, a keep-last-N / keep-best manager, and
sharded optimizer state for ZeRO (`optimizer_state.rank{r}.safetensors`).
"""
from __future__ import annotations

import json
import os
import shutil
import time
from dataclasses import asdict, dataclass, field

import torch

from .serialization import load_safetensors, model_metadata, save_safetensors, to_serde_pretty


@dataclass
class ParamGroupState:
    learning_rate: float = 0.001
    weight_decay: float = 0.0
    momentum: float | None = None
    beta1: float | None = None
    beta2: float | None = None
    epsilon: float | None = None
    step_count: int = 0

    @staticmethod
    def adam(learning_rate, beta1, beta2, epsilon):
        return ParamGroupState(learning_rate, 0.0, None, beta1, beta2, epsilon, 0)

    @staticmethod
    def sgd(learning_rate, momentum, weight_decay):
        return ParamGroupState(learning_rate, weight_decay, momentum, None, None, None, 0)


@dataclass
class OptimizerStateMetadata:
    optimizer_type: str = "Unknown"
    num_param_groups: int = 0
    param_groups: list = field(default_factory=list)


@dataclass
class CheckpointMetadata:
    epoch: int = 0
    global_step: int = 0
    learning_rate: float = 0.0
    train_loss: float | None = None
    val_loss: float | None = None
    best_val_loss: float | None = None
    metrics: dict = field(default_factory=dict)
    optimizer_state: OptimizerStateMetadata = field(default_factory=OptimizerStateMetadata)
    architecture: str = "Sequential"
    model_version: str = "0.1.0"
    timestamp: str = ""
    training_completed: bool = False

    def __post_init__(self):
        if not self.timestamp:
            self.timestamp = str(int(time.time()))

    @staticmethod
    def from_dict(d: dict) -> "CheckpointMetadata":
        d = dict(d)
        os_ = d.pop("optimizer_state", {}) or {}
        groups = [ParamGroupState(**g) for g in os_.get("param_groups", [])]
        md = CheckpointMetadata(**{k: v for k, v in d.items() if k in CheckpointMetadata.__dataclass_fields__})
        md.optimizer_state = OptimizerStateMetadata(os_.get("optimizer_type", "Unknown"),
                                                    os_.get("num_param_groups", len(groups)), groups)
        return md


def _clean(d):
    if isinstance(d, dict):
        return {k: _clean(v) for k, v in d.items()}
    if isinstance(d, list):
        return [_clean(v) for v in d]
    return d


def save_checkpoint(checkpoint_dir, model_params: dict, metadata: CheckpointMetadata,
                    optimizer_moments: dict | None = None, rank: int | None = None) -> None:
    """Write a checkpoint directory. With `rank` set, optimizer moments go to
    optimizer_state.rank{rank}.safetensors (sharded optimizer state) and only
    rank 0 writes the model weights and metadata."""
    os.makedirs(checkpoint_dir, exist_ok=True)
    if rank in (None, 0):
        n = sum(t.numel() for t in model_params.values())
        dt = {torch.float64: "f64", torch.bfloat16: "bf16"}.get(next(iter(model_params.values())).dtype, "f32") \
            if model_params else "f32"
        md = model_metadata(metadata.architecture, dt, n, epoch=metadata.epoch, checkpoint="true")
        save_safetensors(model_params, os.path.join(checkpoint_dir, "model.safetensors"), md)
        with open(os.path.join(checkpoint_dir, "checkpoint_meta.json"), "w") as f:
            f.write(to_serde_pretty(_clean(asdict(metadata))))
    if optimizer_moments:
        name = "optimizer_state.safetensors" if rank is None else f"optimizer_state.rank{rank}.safetensors"
        n = sum(t.numel() for t in optimizer_moments.values())
        save_safetensors(optimizer_moments, os.path.join(checkpoint_dir, name), model_metadata("optimizer", "f32", n))


def load_checkpoint(checkpoint_dir, rank: int | None = None):
    """-> (params, CheckpointMetadata, optimizer moments or None)."""
    if not os.path.isdir(checkpoint_dir):
        raise FileNotFoundError(f"checkpoint directory does not exist: {checkpoint_dir}")
    mp = os.path.join(checkpoint_dir, "model.safetensors")
    if not os.path.exists(mp):
        raise FileNotFoundError(f"model weights not found at {mp}")
    params, _ = load_safetensors(mp)
    with open(os.path.join(checkpoint_dir, "checkpoint_meta.json")) as f:
        meta = CheckpointMetadata.from_dict(json.load(f))
    name = "optimizer_state.safetensors" if rank is None else f"optimizer_state.rank{rank}.safetensors"
    op = os.path.join(checkpoint_dir, name)
    moments = load_safetensors(op)[0] if os.path.exists(op) else None
    return params, meta, moments


def checkpoint_dir_name(epoch: int) -> str:
    return f"checkpoint_epoch_{epoch:04d}"


def list_checkpoints(base_dir) -> list[tuple[int, str]]:
    if not os.path.isdir(base_dir):
        return []
    out = []
    for name in os.listdir(base_dir):
        p = os.path.join(base_dir, name)
        mp = os.path.join(p, "checkpoint_meta.json")
        if os.path.isdir(p) and os.path.exists(mp):
            try:
                with open(mp) as f:
                    out.append((int(json.load(f)["epoch"]), p))
            except (ValueError, KeyError, json.JSONDecodeError):
                continue
    return sorted(out)


def latest_checkpoint(base_dir) -> str | None:
    c = list_checkpoints(base_dir)
    return c[-1][1] if c else None


def best_checkpoint(base_dir) -> str | None:
    best = None
    for _, p in list_checkpoints(base_dir):
        with open(os.path.join(p, "checkpoint_meta.json")) as f:
            v = json.load(f).get("val_loss")
        if v is not None and (best is None or v < best[0]):
            best = (v, p)
    return best[1] if best else None


@dataclass
class CheckpointConfig:
    save_dir: str = "checkpoints"
    keep_last: int = 3
    keep_best: bool = True
    monitor: str = "val_loss"
    mode: str = "min"


class CheckpointManager:
    """Saves epoch checkpoints, keeps the last `keep_last` plus the best one."""

    def __init__(self, config: CheckpointConfig):
        self.config = config
        self.saved: list[str] = []
        self.best_value: float | None = None
        self.best_path: str | None = None

    def save(self, model_params: dict, metadata: CheckpointMetadata, optimizer_moments: dict | None = None) -> str:
        path = os.path.join(self.config.save_dir, checkpoint_dir_name(metadata.epoch))
        save_checkpoint(path, model_params, metadata, optimizer_moments)
        self.saved.append(path)
        v = metadata.val_loss if self.config.monitor == "val_loss" else metadata.metrics.get(self.config.monitor)
        if v is not None and (self.best_value is None or
                              (v < self.best_value if self.config.mode == "min" else v > self.best_value)):
            self.best_value, self.best_path = v, path
        while len(self.saved) > self.config.keep_last:
            old = self.saved.pop(0)
            if self.config.keep_best and old == self.best_path:
                continue
            shutil.rmtree(old, ignore_errors=True)
        return path

    def load_latest(self):
        p = latest_checkpoint(self.config.save_dir)
        return None if p is None else load_checkpoint(p)

    def load_best(self):
        p = self.best_path or best_checkpoint(self.config.save_dir)
        return None if p is None else load_checkpoint(p)
