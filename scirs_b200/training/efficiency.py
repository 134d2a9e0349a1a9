"""Memory-efficient backpropagation, sparse training and progress monitoring.

* `GradientCheckpointManager` keeps copies of chosen layer activations on
  their device within a byte budget (oldest evicted first), chosen by a
  `RecomputationPolicy` (all, none, selective by recomputation cost, every
  n-th layer); `EfficientBackprop.forward_with_checkpoint` runs a layer either
  normally (its activations kept by autograd) or under activation
  recomputation (`torch.utils.checkpoint`: only the input is kept and the
  layer is re-run in the backward), per the same policy, and counts the
  activation bytes that recomputation saved.
* `SparseTraining` keeps the smallest-magnitude fraction `sparsity_ratio` of
  each weight matrix at zero: masks are taken from the weights and re-applied
  after every optimizer step.
* `ProgressMonitor` is a training callback that reports every
  `update_frequency` batches.

Reference parity: scirs2-neural/src/training/backprop_efficient.rs:14-470
(RecomputationPolicy, ActivationCheckpoint, GradientCheckpointManager,
CheckpointStatistics, EfficientBackprop, CpuActivationStore),
sparse_training.rs (SparseTrainingConfig), progress_monitor.rs
(ProgressMonitorConfig).
"""
from __future__ import annotations

import sys
from collections import OrderedDict
from dataclasses import dataclass

import torch
import torch.nn as nn
from torch.utils.checkpoint import checkpoint as _recompute

from .history import Callback


@dataclass(frozen=True)
class RecomputationPolicy:
    """kind: "all" (keep every activation), "none" (recompute everything), "selective" (keep layers
    whose recomputation cost is >= cost_threshold) or "every_n" (keep layers with id % n == 0)."""

    kind: str = "selective"
    cost_threshold: int = 100
    n: int = 1

    def keeps(self, layer_id: int, cost: int) -> bool:
        if self.kind == "all":
            return True
        if self.kind == "none":
            return False
        if self.kind == "selective":
            return cost >= self.cost_threshold
        if self.kind == "every_n":
            return self.n > 0 and layer_id % self.n == 0
        raise ValueError(f"unknown recomputation policy {self.kind!r}")

    @staticmethod
    def checkpoint_all():
        return RecomputationPolicy("all")

    @staticmethod
    def checkpoint_none():
        return RecomputationPolicy("none")

    @staticmethod
    def selective(cost_threshold: int = 100):
        return RecomputationPolicy("selective", cost_threshold=cost_threshold)

    @staticmethod
    def every_n(n: int):
        return RecomputationPolicy("every_n", n=n)


@dataclass
class ActivationCheckpoint:
    layer_id: int
    timestamp: int
    memory_size: int
    recomputation_cost: int
    in_memory: bool = True


@dataclass
class CheckpointStatistics:
    total_checkpoints: int
    in_memory_checkpoints: int
    total_memory: int
    memory_budget: int
    memory_utilization: float


class GradientCheckpointManager:
    def __init__(self, memory_budget: int, policy: RecomputationPolicy | None = None):
        self.budget = int(memory_budget)
        self.policy = policy or RecomputationPolicy()
        self._store: OrderedDict[int, torch.Tensor] = OrderedDict()
        self._meta: dict[int, ActivationCheckpoint] = {}
        self._counter = 0
        self._usage = 0

    def _evict_oldest(self):
        if self._store:
            lid, t = self._store.popitem(last=False)
            self._usage -= t.numel() * t.element_size()
            self._meta[lid].in_memory = False

    def checkpoint_activation(self, layer_id: int, activation: torch.Tensor, recomputation_cost: int) -> bool:
        """Store a device copy of `activation` if the policy keeps this layer; returns whether it did."""
        if not self.policy.keeps(layer_id, recomputation_cost):
            return False
        size = activation.numel() * activation.element_size()
        if size > self.budget:
            return False
        if layer_id in self._store:
            self.remove_checkpoint(layer_id)
        while self._usage + size > self.budget and self._store:
            self._evict_oldest()
        self._store[layer_id] = activation.detach().clone()
        self._meta[layer_id] = ActivationCheckpoint(layer_id, self._counter, size, recomputation_cost)
        self._counter += 1
        self._usage += size
        return True

    def get_checkpoint(self, layer_id: int) -> torch.Tensor | None:
        """Return and remove the stored activation of `layer_id` (None if not stored)."""
        t = self._store.pop(layer_id, None)
        if t is not None:
            self._usage -= t.numel() * t.element_size()
            self._meta[layer_id].in_memory = False
        return t

    def has_checkpoint(self, layer_id: int) -> bool:
        return layer_id in self._store

    def remove_checkpoint(self, layer_id: int):
        self.get_checkpoint(layer_id)

    def clear(self):
        for lid in list(self._store):
            self.get_checkpoint(lid)

    def memory_usage(self) -> int:
        return self._usage

    def memory_budget(self) -> int:
        return self.budget

    def num_checkpoints(self) -> int:
        return len(self._store)

    def get_statistics(self) -> CheckpointStatistics:
        return CheckpointStatistics(len(self._meta), len(self._store), self._usage, self.budget,
                                    self._usage / self.budget if self.budget else 0.0)


class EfficientBackprop:
    def __init__(self, memory_budget: int, policy: RecomputationPolicy | None = None, enabled: bool = True):
        self.manager = GradientCheckpointManager(memory_budget, policy)
        self.enabled = enabled
        self.recomputed_bytes = 0  # activation bytes that recomputation did not keep (estimated from outputs)

    def forward_with_checkpoint(self, layer_id: int, x: torch.Tensor, forward_fn, recomputation_cost: int = 0):
        """Run forward_fn(x). If enabled and the policy keeps the layer, its input is also stored in the
        manager and autograd keeps the activations; otherwise the layer runs under activation
        recomputation (only the input is saved, the forward re-runs in the backward)."""
        if not self.enabled or not torch.is_grad_enabled():
            return forward_fn(x)
        if self.manager.checkpoint_activation(layer_id, x, recomputation_cost):
            return forward_fn(x)
        y = _recompute(forward_fn, x, use_reentrant=False)
        self.recomputed_bytes += y.numel() * y.element_size()
        return y

    def set_enabled(self, enabled: bool):
        self.enabled = enabled

    def is_enabled(self) -> bool:
        return self.enabled

    def checkpoint_manager(self) -> GradientCheckpointManager:
        return self.manager

    def get_statistics(self) -> CheckpointStatistics:
        return self.manager.get_statistics()

    def clear_checkpoints(self):
        self.manager.clear()


# ---------------------------------------------------------------------------- sparse training
@dataclass
class SparseTrainingConfig:
    enabled: bool = False
    sparsity_ratio: float = 0.0


class SparseTraining:
    """Magnitude masks on every >= 2-D parameter of `model` (the smallest |w| fraction set to zero),
    recomputed by `update_masks` and re-applied by `apply` (call after each optimizer step)."""

    def __init__(self, model: nn.Module, config: SparseTrainingConfig):
        if not 0.0 <= config.sparsity_ratio < 1.0:
            raise ValueError("sparsity_ratio must be in [0, 1)")
        self.model, self.config = model, config
        self.masks: dict[str, torch.Tensor] = {}
        if config.enabled:
            self.update_masks()
            self.apply()

    @torch.no_grad()
    def update_masks(self):
        self.masks = {}
        for name, p in self.model.named_parameters():
            if p.dim() < 2 or self.config.sparsity_ratio <= 0:
                continue
            k = int(p.numel() * self.config.sparsity_ratio)
            if k == 0:
                continue
            thresh = p.detach().abs().flatten().kthvalue(k).values
            self.masks[name] = (p.detach().abs() > thresh).to(p.dtype)

    @torch.no_grad()
    def apply(self):
        if not self.config.enabled:
            return
        params = dict(self.model.named_parameters())
        for name, m in self.masks.items():
            params[name].mul_(m)

    def sparsity(self) -> float:
        tot = sum(m.numel() for m in self.masks.values())
        return 0.0 if tot == 0 else 1.0 - sum(float(m.sum()) for m in self.masks.values()) / tot


# ---------------------------------------------------------------------------- progress monitor
@dataclass
class ProgressMonitorConfig:
    show_progress: bool = True
    update_frequency: int = 1


class ProgressMonitor(Callback):
    def __init__(self, config: ProgressMonitorConfig | None = None, stream=None):
        self.config = config or ProgressMonitorConfig()
        self.stream = stream if stream is not None else sys.stderr
        self.reports: list[str] = []

    def on_batch_end(self, step, model, logs=None):
        if not self.config.show_progress or self.config.update_frequency <= 0:
            return
        if (step + 1) % self.config.update_frequency == 0:
            items = ", ".join(f"{k}={v:.4g}" if isinstance(v, float) else f"{k}={v}" for k, v in (logs or {}).items())
            line = f"step {step + 1}" + (f": {items}" if items else "")
            self.reports.append(line)
            print(line, file=self.stream)
