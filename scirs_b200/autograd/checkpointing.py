"""Activation checkpointing (recompute in backward) and placement plans.

Plans pick which layer inputs of an n-layer chain are stored; the layers
between two stored points are re-run during backward:
  uniform(k)   every k-th layer (+ the last)
  sqrt         uniform with k = ceil(sqrt(n)): O(sqrt n) memory and recompute
  binomial(b)  Revolve-style for a budget of b stored activations: t is the
               least number of forward sweeps with C(t+b, b) >= n, and the
               chain is split recursively so that the left part of a
               segment with s slots and t sweeps holds C(t-1+s, s) layers
               (the most that s slots can cover with one sweep fewer)

`checkpoint_sequential(layers, x, plan)` runs a layer list under a plan with
torch.utils.checkpoint (non-reentrant), so the recomputation reproduces the
forward exactly (RNG state included).

Reference parity: scirs2-autograd/src/autodiff_enhanced.rs:20-240
(CheckpointStrategy, CheckpointPlan, sqrt/binomial/uniform plans) and
tensor_ops/checkpoint_ops.rs:67-606 (checkpoint, checkpoint_segment).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
from torch.utils.checkpoint import checkpoint as _ckpt


@dataclass
class CheckpointPlan:
    num_layers: int
    checkpoint_indices: list = field(default_factory=list)
    strategy: str = "none"
    peak_memory: int = 0
    recomputation_cost: int = 0


def uniform_checkpoint_plan(num_layers: int, interval: int) -> CheckpointPlan:
    k = max(1, interval)
    idx = list(range(0, num_layers, k))
    if num_layers and idx[-1] != num_layers - 1:
        idx.append(num_layers - 1)
    return CheckpointPlan(num_layers, idx, f"uniform({k})", len(idx) + k, (len(idx) - 1) * k if len(idx) > 1 else 0)


def sqrt_checkpoint_plan(num_layers: int) -> CheckpointPlan:
    if num_layers == 0:
        return CheckpointPlan(0, [], "sqrt")
    p = uniform_checkpoint_plan(num_layers, math.ceil(math.sqrt(num_layers)))
    p.strategy = "sqrt"
    return p


def _revolve_sweeps(n: int, b: int) -> int:
    t = 0
    while math.comb(t + b, b) < n:
        t += 1
    return t


def binomial_checkpoint_plan(num_layers: int, memory_budget: int) -> CheckpointPlan:
    n, b = num_layers, min(memory_budget, num_layers)
    if n == 0 or b == 0:
        return CheckpointPlan(n, [], f"binomial({memory_budget})")
    t = _revolve_sweeps(n, b)
    idx: set[int] = set()

    def place(lo: int, length: int, slots: int, sweeps: int):
        if length <= 1 or slots <= 0:
            return
        idx.add(lo)
        if slots == 1 or sweeps == 0:
            return
        left = min(max(1, math.comb(sweeps - 1 + slots, slots)), length - 1)
        place(lo, left, slots, sweeps - 1)
        place(lo + left, length - left, slots - 1, sweeps)

    place(0, n, b, t)
    idx.add(0)
    out = sorted(idx)[:max(b, 1)]
    return CheckpointPlan(n, out, f"binomial({memory_budget})", b, t)


def checkpoint(fn, *args, **kwargs):
    """Run `fn(*args)` without storing its internal activations; they are
    recomputed during backward."""
    return _ckpt(fn, *args, use_reentrant=False, **kwargs)


def checkpoint_segment(fn, *tensors):
    return checkpoint(fn, *tensors)


def checkpoint_sequential(layers, x, plan: CheckpointPlan | None = None):
    """Run `layers` in order; each stretch between consecutive checkpoint
    indices of `plan` (default: sqrt plan) is one recomputed segment."""
    layers = list(layers)
    plan = plan or sqrt_checkpoint_plan(len(layers))
    bounds = sorted(set(plan.checkpoint_indices) | {0}) + [len(layers)]
    for a, b in zip(bounds[:-1], bounds[1:]):
        if b <= a:
            continue
        seg = layers[a:b]

        def run(h, seg=seg):
            for m in seg:
                h = m(h)
            return h

        x = checkpoint(run, x) if torch.is_grad_enabled() else run(x)
    return x
