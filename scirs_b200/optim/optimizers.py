"""Optimizers for ordinary torch parameters: SGD, Adam, AdamW, RMSprop, Adagrad.

On the first step (or at construction) the parameters are re-homed into one
flat buffer (parameters become views of it) and their gradients into one flat
gradient buffer that autograd accumulates into in place, so each `step()` is
a single fused launch of the optimizer kernel (scirs_b200/csrc/optim.cu) —
on GPU — or its PyTorch reference on CPU. bf16 parameters keep an fp32
master copy inside the optimizer.

Update rules are the reference's (scirs2-neural/src/optimizers/*.rs, cited
in optim.cu); the API follows torch.optim (step / zero_grad / state_dict)
plus the reference's `get_learning_rate` / `set_learning_rate`.
"""
from __future__ import annotations

import torch

from ..ops import kernels as K

_ALIGN = 64


class FlatOptimizer:
    mode = "adamw"

    def __init__(self, params, lr=1e-3, *, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, momentum=0.0,
                 rho=0.9, max_grad_norm=0.0, grad_multiplier=1.0):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("optimizer got an empty parameter list")
        self.lr, self.beta1, self.beta2, self.eps = lr, beta1, beta2, eps
        self.weight_decay, self.momentum, self.rho = weight_decay, momentum, rho
        self.max_grad_norm, self.grad_multiplier = max_grad_norm, grad_multiplier
        self.t = 0
        self._build()

    # ------------------------------------------------------------------ storage
    def _build(self):
        ps = self.params
        dev, dt = ps[0].device, ps[0].dtype
        if any(p.device != dev or p.dtype != dt for p in ps):
            raise ValueError("all parameters of one optimizer must share device and dtype")
        offs, n = [], 0
        for p in ps:
            offs.append(n)
            n += (p.numel() + _ALIGN - 1) // _ALIGN * _ALIGN
        self.n, self.device, self.dtype = n, dev, dt
        flat = torch.zeros(n, dtype=dt, device=dev)
        gflat = torch.zeros(n, dtype=dt, device=dev)
        with torch.no_grad():
            for p, o in zip(ps, offs):
                flat[o : o + p.numel()].copy_(p.reshape(-1))
                p.data = flat[o : o + p.numel()].view_as(p)
                p.grad = gflat[o : o + p.numel()].view_as(p)
        self.flat, self.gflat, self.offs = flat, gflat, offs
        if dt == torch.float32:
            self.master, self.p16 = flat, None
        else:
            self.master, self.p16 = flat.float(), flat
        need2 = self.mode in ("adam", "adamw")
        need1 = need2 or self.mode in ("rmsprop", "adagrad") or (self.mode == "sgd" and self.momentum > 0)
        self.s1 = torch.zeros(n if need1 else 0, dtype=torch.float32, device=dev)
        self.s2 = torch.zeros(n if need2 else 0, dtype=torch.float32, device=dev)
        self.hp = torch.zeros(16, dtype=torch.float32, device=dev)
        self.part = torch.zeros(1024, dtype=torch.float32, device=dev) if self.max_grad_norm > 0 else None
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=dev)

    def _check_views(self):
        # Re-attach gradients that user code replaced (e.g. zero_grad(set_to_none=True) from elsewhere).
        for p, o in zip(self.params, self.offs):
            g = p.grad
            if g is None or g.data_ptr() != self.gflat[o:].data_ptr():
                view = self.gflat[o : o + p.numel()].view_as(p)
                if g is not None:
                    view.copy_(g)
                else:
                    view.zero_()
                p.grad = view

    # ------------------------------------------------------------------ API
    def zero_grad(self, set_to_none: bool = False):
        self.gflat.zero_()

    def get_learning_rate(self):
        return self.lr

    def set_learning_rate(self, lr):
        self.lr = lr

    @torch.no_grad()
    def step(self):
        self._check_views()
        self.t += 1
        b1 = {"sgd": self.momentum, "rmsprop": self.rho}.get(self.mode, self.beta1)
        bc1 = 1.0 - self.beta1**self.t
        bc2 = 1.0 - self.beta2**self.t
        vals = [self.lr, b1, self.beta2, self.eps, self.weight_decay, bc1, bc2, self.grad_multiplier,
                self.max_grad_norm]
        self.hp[: len(vals)] = torch.tensor(vals, dtype=torch.float32)
        K.optim_step(self.mode, self.master, self.s1, self.s2, self.gflat, self.p16, self.n, self.hp,
                     part=self.part, norm_out=self.grad_norm if self.part is not None else None)

    def state_dict(self):
        return {"t": self.t, "lr": self.lr, "s1": self.s1.clone(), "s2": self.s2.clone(), "master": self.master.clone()}

    def load_state_dict(self, sd):
        self.t, self.lr = int(sd["t"]), float(sd["lr"])
        self.s1.copy_(sd["s1"])
        self.s2.copy_(sd["s2"])
        self.master.copy_(sd["master"])
        if self.p16 is not None:
            self.p16.copy_(self.master)

    @property
    def param_groups(self):  # minimal torch-style view for schedulers
        return [{"lr": self.lr, "params": self.params}]


class SGD(FlatOptimizer):
    """p -= v, v = momentum v + lr (g + wd p) (scirs2-neural/src/optimizers/sgd.rs:95-130)."""

    mode = "sgd"

    def __init__(self, params, lr=0.01, momentum=0.0, weight_decay=0.0, **kw):
        super().__init__(params, lr, momentum=momentum, weight_decay=weight_decay, **kw)


class Adam(FlatOptimizer):
    """Adam with L2 weight decay added to the gradient (adam.rs:163-215)."""

    mode = "adam"

    def __init__(self, params, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, **kw):
        super().__init__(params, lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay, **kw)


class AdamW(FlatOptimizer):
    """Adam with decoupled weight decay p *= 1 - lr wd (adamw.rs:149-196)."""

    mode = "adamw"

    def __init__(self, params, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, **kw):
        super().__init__(params, lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay, **kw)


class RMSprop(FlatOptimizer):
    """v = rho v + (1-rho) g^2; p -= lr g / (sqrt v + eps) (rmsprop.rs:123-161)."""

    mode = "rmsprop"

    def __init__(self, params, lr=1e-3, rho=0.9, eps=1e-8, weight_decay=0.0, **kw):
        super().__init__(params, lr, rho=rho, eps=eps, weight_decay=weight_decay, **kw)


class Adagrad(FlatOptimizer):
    """s += g^2; p -= lr g / (sqrt s + eps) (adagrad.rs:100-130)."""

    mode = "adagrad"

    def __init__(self, params, lr=1e-2, eps=1e-10, weight_decay=0.0, **kw):
        super().__init__(params, lr, eps=eps, weight_decay=weight_decay, **kw)


def get_optimizer(name, params, learning_rate=None, **kw):
    if not isinstance(name, str):
        return name
    table = {"sgd": SGD, "adam": Adam, "adamw": AdamW, "rmsprop": RMSprop, "adagrad": Adagrad}
    cls = table[name.lower()]
    if learning_rate is not None:
        kw["lr"] = learning_rate
    return cls(params, **kw)
