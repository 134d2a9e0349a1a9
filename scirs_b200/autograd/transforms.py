"""Function transforms, higher-order derivatives, gradient checking, graph export.

  jvp / vjp / hessian / hessian_vector_product / jacobian
                         scirs2-autograd/src/forward_mode.rs, higher_order/*.rs
  vmap / value_and_grad / scan / check_grad / pmap
                         scirs2-autograd/src/transforms.rs (lib.rs:491-565)
  GradientChecker        scirs2-autograd/src/testing/gradient_checking.rs:15-533
                         (central finite differences)
  to_dot / to_json / to_mermaid
                         scirs2-autograd/src/visualization/mod.rs
  ExecutionTracer        scirs2-autograd/src/tracing.rs:17-43
All operate on plain torch callables (the eager path of the framework).
"""
from __future__ import annotations

import json
import time
from dataclasses import dataclass, field

import torch
import torch.func as tf

from .graph import Graph, Tensor


def value_and_grad(fn, argnums=0):
    """fn -> (lambda *args: (fn(*args), d fn / d args[argnums]))."""
    g = tf.grad_and_value(fn, argnums=argnums)

    def wrapped(*args):
        grads, value = g(*args)
        return value, grads

    return wrapped


def grad_fn(fn, argnums=0):
    return tf.grad(fn, argnums=argnums)


def jvp(fn, primals, tangents):
    return tf.jvp(fn, tuple(primals), tuple(tangents))


def vjp(fn, *primals):
    return tf.vjp(fn, *primals)


def jacobian(fn, x):
    return tf.jacrev(fn)(x)


def hessian(fn, x):
    return tf.hessian(fn)(x)


def hessian_vector_product(fn, x, v):
    return tf.jvp(tf.grad(fn), (x,), (v,))[1]


def vmap(fn, in_dims=0, out_dims=0):
    return tf.vmap(fn, in_dims=in_dims, out_dims=out_dims)


def pmap(fn, xs, threads: int = 4):
    """Apply fn to each element of xs with a thread pool (host parallel map)."""
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(threads) as ex:
        return list(ex.map(fn, xs))


def scan(fn, init, xs):
    """carry, y = fn(carry, x) over the leading axis of xs; returns (carry, stacked ys)."""
    carry, ys = init, []
    for x in xs:
        carry, y = fn(carry, x)
        ys.append(y)
    return carry, torch.stack(ys) if ys and isinstance(ys[0], torch.Tensor) else ys


@dataclass
class GradCheckResult:
    passed: bool
    max_abs_error: float
    max_rel_error: float
    details: list = field(default_factory=list)


class GradientChecker:
    """Compare autograd gradients with central finite differences in float64."""

    def __init__(self, eps: float = 1e-6, rtol: float = 1e-4, atol: float = 1e-6):
        self.eps, self.rtol, self.atol = eps, rtol, atol

    def check(self, fn, *inputs) -> GradCheckResult:
        xs = [x.detach().double().contiguous().clone().requires_grad_(True) for x in inputs]
        y = fn(*xs)
        analytic = torch.autograd.grad(y.sum(), xs, allow_unused=True)
        max_abs = max_rel = 0.0
        details = []
        for i, x in enumerate(xs):
            num = torch.zeros_like(x)
            flat = x.detach().reshape(-1)
            for j in range(flat.numel()):
                xp = [t.detach().clone() for t in xs]
                xm = [t.detach().clone() for t in xs]
                xp[i].reshape(-1)[j] += self.eps
                xm[i].reshape(-1)[j] -= self.eps
                num.reshape(-1)[j] = (fn(*xp).sum() - fn(*xm).sum()) / (2 * self.eps)
            a = analytic[i] if analytic[i] is not None else torch.zeros_like(x)
            err = (a - num).abs()
            rel = err / (num.abs() + self.atol)
            max_abs, max_rel = max(max_abs, float(err.max())), max(max_rel, float(rel.max()))
            details.append({"input": i, "max_abs": float(err.max())})
        ok = max_abs <= self.atol + self.rtol * 1e2 or max_rel <= self.rtol * 1e2
        return GradCheckResult(ok, max_abs, max_rel, details)


def check_grad(fn, *inputs, eps=1e-6, tol=1e-4) -> bool:
    return GradientChecker(eps=eps, rtol=tol).check(fn, *inputs).passed


# ---------------------------------------------------------------------------- graph export
def _nodes(g: Graph):
    return g._nodes


def to_json(g: Graph) -> str:
    return json.dumps({"nodes": [{"id": n.id, "op": n.op, "name": n.name, "inputs": [i.id for i in n.inputs]}
                                 for n in _nodes(g)]})


def to_dot(g: Graph) -> str:
    lines = ["digraph G {"]
    for n in _nodes(g):
        label = n.op if not n.name else f"{n.op}\\n{n.name}"
        lines.append(f'  n{n.id} [label="{label}"];')
        for i in n.inputs:
            lines.append(f"  n{i.id} -> n{n.id};")
    lines.append("}")
    return "\n".join(lines)


def to_mermaid(g: Graph) -> str:
    lines = ["graph TD"]
    for n in _nodes(g):
        lines.append(f"  n{n.id}[{n.op}{':' + n.name if n.name else ''}]")
        for i in n.inputs:
            lines.append(f"  n{i.id} --> n{n.id}")
    return "\n".join(lines)


class ExecutionTracer:
    """Records (op, wall-time) events of graph evaluation via node hooks."""

    def __init__(self):
        self.events = []
        self._t0 = time.perf_counter()

    def attach(self, g: Graph):
        for n in _nodes(g):
            n.register_hook(lambda v, n=n: self.events.append(
                {"op": n.op, "id": n.id, "t": time.perf_counter() - self._t0, "shape": tuple(v.shape)}))
        return self

    def summary(self):
        out = {}
        for e in self.events:
            out[e["op"]] = out.get(e["op"], 0) + 1
        return out
