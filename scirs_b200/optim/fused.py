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

    def _hp_values(self):
        b1, b2 = self.betas
        if self.mode == "sgd":
            b1 = self.momentum
        elif self.mode == "rmsprop":
            b1 = self.rho
        return [self.lr, b1, b2, self.eps, self.weight_decay, 1.0, 1.0, self.grad_multiplier, self.max_grad_norm]

    def _hyper(self):
        """Upload hyperparameters when they changed. The step counter and the
        bias corrections are maintained on the device (hp[9], hp[10] = 1), so a
        step captured in a CUDA graph replays correctly without host writes."""
        self.t += 1
        vals = self._hp_values()
        if getattr(self, "_uploaded", None) != vals:
            self._hp_host[: len(vals)] = torch.tensor(vals, dtype=torch.float32)
            self._hp_host[9] = float(self.t - 1)  # incremented on the device before use
            self._hp_host[10] = 1.0
            if getattr(self, "_uploaded", None) is not None:
                # keep the device step counter: only the first upload sets it
                torch.cuda.current_stream().synchronize() if self.hp.is_cuda else None
                self._hp_host[9] = float(self.hp[9].item())
            self.hp.copy_(self._hp_host, non_blocking=False)
            self._uploaded = vals

    def set_lr(self, lr: float):
        self.lr = lr

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
        self.hp[9] = float(self.t)
        self._uploaded = None
