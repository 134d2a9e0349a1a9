"""Fused single-launch optimizers over a flat parameter buffer.

The update rules are those of the reference optimizers (see
scirs_b200/csrc/optim.cu for the per-rule citations). The step-dependent
scalars live in a small device tensor that is refreshed from the host before
each step, so the same launch can be captured once in a CUDA graph and
replayed every step.
"""
from __future__ import annotations

import torch

from ..ops import kernels as K
from ..utils.flat import FlatParams


class FusedFlatOptimizer:
    """Adam / AdamW / SGD / RMSprop / Adagrad over a :class:`FlatParams`.

    Global-norm gradient clipping (`max_grad_norm`), a gradient multiplier
    (e.g. 1/loss_scale for mixed precision) and skipping a step whose
    gradient norm is not finite are folded into the same launch.
    """

    def __init__(
        self,
        flat: FlatParams,
        mode: str = "adamw",
        lr: float = 1e-3,
        betas=(0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.0,
        momentum: float = 0.0,
        rho: float = 0.9,
        max_grad_norm: float = 0.0,
        grad_multiplier: float = 1.0,
    ):
        self.flat = flat
        self.mode = mode
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.momentum = momentum
        self.rho = rho
        self.max_grad_norm = max_grad_norm
        self.grad_multiplier = grad_multiplier
        self.t = 0
        dev = flat.master.device
        n = flat.total
        need2 = mode in ("adam", "adamw")
        need1 = need2 or mode in ("rmsprop", "adagrad") or (mode == "sgd" and momentum > 0)
        self.state1 = torch.zeros(n if need1 else 0, dtype=torch.float32, device=dev)
        self.state2 = torch.zeros(n if need2 else 0, dtype=torch.float32, device=dev)
        self.hp = torch.zeros(16, dtype=torch.float32, device=dev)
        self._hp_host = torch.zeros(16, dtype=torch.float32, pin_memory=dev.type == "cuda")
        self.part = torch.zeros(1024, dtype=torch.float32, device=dev)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.launches_per_step = 2

    def _hyper(self):
        self.t += 1
        b1, b2 = self.betas
        if self.mode == "sgd":
            b1 = self.momentum
        elif self.mode == "rmsprop":
            b1 = self.rho
        bc1 = 1.0 - self.betas[0] ** self.t
        bc2 = 1.0 - self.betas[1] ** self.t
        vals = [self.lr, b1, b2, self.eps, self.weight_decay, bc1, bc2, self.grad_multiplier, self.max_grad_norm]
        self._hp_host[: len(vals)] = torch.tensor(vals, dtype=torch.float32)
        self.hp.copy_(self._hp_host, non_blocking=True)

    def step(self):
        self._hyper()
        f = self.flat
        K.optim_step(
            self.mode,
            f.master,
            self.state1,
            self.state2,
            f.grad,
            f.p16,
            f.total,
            self.hp,
            part=self.part,
            norm_out=self.grad_norm,
            decay_mask=f.decay_mask,
        )

    def state_dict(self):
        return {"t": self.t, "state1": self.state1.clone(), "state2": self.state2.clone(), "lr": self.lr}

    def load_state_dict(self, sd):
        self.t = int(sd["t"])
        self.state1.copy_(sd["state1"])
        self.state2.copy_(sd["state2"])
        self.lr = sd.get("lr", self.lr)
