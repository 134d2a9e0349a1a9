"""Variable store and graph-level optimizers.

  VariableEnvironment   scirs2-autograd/src/variable.rs:154-955 (namespaced
                        variables, `name(..).set(..)`, JSON save/load with the
                        reference's {"array_list": [...], "name_to_id": {...}}
                        layout, arrays in ndarray's serde form {"v": 1, "dim", "data"})
  Adam / AdamW / SGD / MomentumSGD / AdaGrad
                        scirs2-autograd/src/optimizers/*.rs: `update(vars, grads, ctx, feeder)`
                        evaluates the gradient nodes and writes the new values
                        back into the environment (one fused kernel launch per
                        update on GPU-resident variables).
"""
from __future__ import annotations

import json

import numpy as np
import torch

from ..ops import kernels as K
from . import graph as G


class _NameRef:
    def __init__(self, env, name):
        self.env, self.name_ = env, name

    def set(self, value):
        return self.env.set(self.name_, value)

    def id(self):
        return self.env.name_to_id[self.name_]


class VariableEnvironment:
    def __init__(self, device=None, dtype=torch.float32):
        self.array_list: list[torch.Tensor] = []
        self.name_to_id: dict[str, int] = {}
        self.device, self.dtype = device, dtype
        self._prefix = ""

    # ------------------------------------------------------------ creation
    def name(self, name: str) -> _NameRef:
        return _NameRef(self, self._prefix + name)

    def namespace(self, ns: str) -> "VariableEnvironment":
        view = VariableEnvironment.__new__(VariableEnvironment)
        view.__dict__ = self.__dict__.copy()
        view._prefix = self._prefix + ns + "/"
        # share the storage
        view.array_list, view.name_to_id = self.array_list, self.name_to_id
        return view

    def set(self, name_or_value, value=None) -> int:
        if value is None:
            name, value = None, name_or_value
        else:
            name = name_or_value
        t = torch.as_tensor(np.asarray(value) if not isinstance(value, torch.Tensor) else value)
        t = t.to(device=self.device, dtype=self.dtype if t.is_floating_point() else t.dtype).clone()
        if name is not None and name in self.name_to_id:
            vid = self.name_to_id[name]
            self.array_list[vid] = t
            return vid
        self.array_list.append(t)
        vid = len(self.array_list) - 1
        if name is not None:
            self.name_to_id[name] = vid
        return vid

    def resolve(self, name_or_id) -> int:
        if isinstance(name_or_id, int):
            return name_or_id
        key = name_or_id if name_or_id in self.name_to_id else self._prefix + name_or_id
        return self.name_to_id[key]

    def array(self, vid) -> torch.Tensor:
        return self.array_list[self.resolve(vid)]

    def get_array_by_name(self, name):
        return self.array(name).detach().cpu().numpy()

    def iter(self):
        return enumerate(self.array_list)

    def default_namespace(self):
        return self

    # ------------------------------------------------------------ graphs
    def run(self, fn):
        """Create a graph bound to this environment and call fn(ctx)."""
        return G.run(fn, env=self)

    # ------------------------------------------------------------ persistence
    def save(self, path) -> None:
        obj = {
            "array_list": [
                {"v": 1, "dim": list(t.shape), "data": [float(x) for x in t.detach().cpu().double().reshape(-1)]}
                for t in self.array_list
            ],
            "name_to_id": dict(self.name_to_id),
        }
        with open(path, "w") as f:
            json.dump(obj, f)

    @staticmethod
    def load(path, device=None, dtype=torch.float32) -> "VariableEnvironment":
        with open(path) as f:
            obj = json.load(f)
        env = VariableEnvironment(device=device, dtype=dtype)
        for a in obj["array_list"]:
            env.array_list.append(torch.tensor(a["data"], dtype=dtype, device=device).reshape(a["dim"]))
        env.name_to_id = {k: int(v) for k, v in obj["name_to_id"].items()}
        return env

    def initialize(self, path):
        other = VariableEnvironment.load(path, self.device, self.dtype)
        self.array_list, self.name_to_id = other.array_list, other.name_to_id


# ============================================================================ optimizers
class Optimizer:
    mode = "sgd"

    def __init__(self, var_ids, env: VariableEnvironment, lr=1e-3, **hp):
        self.env = env
        self.var_ids = [env.resolve(v) for v in var_ids]
        self.lr, self.hp, self.t = lr, hp, 0
        self.s1 = {v: torch.zeros_like(env.array(v), dtype=torch.float32) for v in self.var_ids}
        self.s2 = {v: torch.zeros_like(env.array(v), dtype=torch.float32) for v in self.var_ids}

    @classmethod
    def default(cls, name, var_ids, env):
        return cls(var_ids, env)

    def update(self, variables, grads, ctx: G.Graph, feeder: G.Feeder | None = None):
        """Evaluate `grads` (graph nodes aligned with `variables`) and apply one step."""
        ev = ctx.evaluator().torch().extend(grads)
        if feeder is not None:
            ev.set_feeder(feeder)
        gvals = ev.run()
        self.apply_gradients([v.attrs["vid"] for v in variables], gvals)

    @torch.no_grad()
    def apply_gradients(self, vids, gvals):
        self.t += 1
        b1 = self.hp.get("beta1", self.hp.get("momentum", 0.9))
        b2 = self.hp.get("beta2", 0.999)
        hp = torch.tensor([self.lr, b1, b2, self.hp.get("eps", 1e-8), self.hp.get("weight_decay", 0.0),
                           1 - self.hp.get("beta1", 0.9) ** self.t, 1 - b2**self.t, 1.0, 0.0], dtype=torch.float32)
        for vid, g in zip(vids, gvals):
            p = self.env.array_list[vid]
            p32 = p.float().reshape(-1).contiguous()
            hpd = hp.to(p32.device)
            K.optim_step(self.mode, p32, self.s1[vid].reshape(-1), self.s2[vid].reshape(-1),
                         g.float().reshape(-1).contiguous(), None, p32.numel(), hpd)
            self.env.array_list[vid] = p32.reshape(p.shape).to(p.dtype)


class SGD(Optimizer):
    mode = "sgd"

    def __init__(self, var_ids, env, lr=0.01, momentum=0.0):
        super().__init__(var_ids, env, lr, momentum=momentum)


class MomentumSGD(SGD):
    def __init__(self, var_ids, env, lr=0.01, momentum=0.9):
        super().__init__(var_ids, env, lr, momentum)


class Adam(Optimizer):
    mode = "adam"

    def __init__(self, var_ids, env, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0):
        super().__init__(var_ids, env, lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay)


class AdamW(Optimizer):
    mode = "adamw"

    def __init__(self, var_ids, env, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01):
        super().__init__(var_ids, env, lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay)


class AdaGrad(Optimizer):
    mode = "adagrad"

    def __init__(self, var_ids, env, lr=1e-2, eps=1e-10):
        super().__init__(var_ids, env, lr, eps=eps)
