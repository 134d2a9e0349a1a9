"""Define-then-run autodiff graphs.

The graph API of the reference's autograd crate (scirs2-autograd/src/graph.rs:21-473,
tensor.rs:54-215, evaluation.rs:56-212, variable.rs:154-955):

    env = VariableEnvironment()
    env.name("w").set(array)
    def body(ctx):
        x = ctx.placeholder("x", [-1, 784])
        w = ctx.variable("w")
        loss = T.reduce_mean(T.square(T.matmul(x, w)))
        g, = T.grad([loss], [w])
        return ctx.evaluator().push(loss).push(g).feed(x, data).run()
    env.run(body)

Nodes are lazy; evaluation walks the graph once per `Evaluator.run` with
memoisation. Gradients are graph nodes too (so grad-of-grad works): the
forward values are computed as differentiable torch tensors and each `grad`
node calls torch.autograd.grad with create_graph=True. Compute runs on the
device of the fed/variable tensors (CUDA bf16 matmuls go through the
framework's tensor-core GEMM via :mod:`scirs_b200.autograd.ops`).
"""
from __future__ import annotations

import itertools

import numpy as np
import torch

_ids = itertools.count()


class Tensor:
    """A lazy node of a graph (reference: scirs2-autograd/src/tensor.rs)."""

    __slots__ = ("graph", "op", "inputs", "attrs", "id", "name", "shape_hint", "hooks")

    def __init__(self, graph, op: str, inputs=(), attrs=None, name=None, shape_hint=None):
        self.graph = graph
        self.op = op
        self.inputs = tuple(inputs)
        self.attrs = attrs or {}
        self.id = next(_ids)
        self.name = name
        self.shape_hint = shape_hint
        self.hooks = []
        graph._nodes.append(self)
        if len(graph._nodes) in (50_000, 500_000):
            import warnings

            warnings.warn(f"graph has {len(graph._nodes)} nodes")

    # ------------------------------------------------------------ evaluation
    def eval(self, feeds=None):
        ev = self.graph.evaluator().push(self)
        for k, v in (feeds or {}).items():
            ev.feed(k, v)
        return ev.run()[0]

    # ------------------------------------------------------------ hooks
    def register_hook(self, fn):
        """fn(value) is called with this node's value each time it is evaluated."""
        self.hooks.append(fn)
        return self

    def show(self, prefix: str = ""):
        return self.register_hook(lambda v: print(prefix, v))

    def raw_hook(self, fn):
        return self.register_hook(fn)

    # ------------------------------------------------------------ operators
    def _c(self, other):
        return other if isinstance(other, Tensor) else self.graph.constant(other)

    def __add__(self, o):
        return Tensor(self.graph, "add", (self, self._c(o)))

    __radd__ = __add__

    def __sub__(self, o):
        return Tensor(self.graph, "sub", (self, self._c(o)))

    def __rsub__(self, o):
        return Tensor(self.graph, "sub", (self._c(o), self))

    def __mul__(self, o):
        return Tensor(self.graph, "mul", (self, self._c(o)))

    __rmul__ = __mul__

    def __truediv__(self, o):
        return Tensor(self.graph, "div", (self, self._c(o)))

    def __rtruediv__(self, o):
        return Tensor(self.graph, "div", (self._c(o), self))

    def __neg__(self):
        return Tensor(self.graph, "neg", (self,))

    def __matmul__(self, o):
        return Tensor(self.graph, "matmul", (self, self._c(o)))

    def __pow__(self, p):
        return Tensor(self.graph, "pow", (self,), {"p": p})

    def __getitem__(self, idx):
        return Tensor(self.graph, "getitem", (self,), {"idx": idx})

    def __repr__(self):
        return f"Tensor(id={self.id}, op={self.op}{', name=' + self.name if self.name else ''})"


class Graph:
    """Arena of nodes (one per `run` scope)."""

    def __init__(self, env=None):
        self._nodes: list[Tensor] = []
        self.env = env
        self.device = None
        self.dtype = torch.float32

    # ------------------------------------------------------------ sources
    def placeholder(self, name: str, shape=None) -> Tensor:
        return Tensor(self, "placeholder", (), {"name": name}, name=name, shape_hint=shape)

    def variable(self, name_or_id) -> Tensor:
        if self.env is None:
            raise RuntimeError("no VariableEnvironment bound to this graph")
        vid = self.env.resolve(name_or_id)
        return Tensor(self, "variable", (), {"vid": vid}, name=str(name_or_id))

    def constant(self, value) -> Tensor:
        return Tensor(self, "constant", (), {"value": value})

    def zeros(self, shape) -> Tensor:
        return Tensor(self, "zeros", (), {"shape": tuple(shape)})

    def ones(self, shape) -> Tensor:
        return Tensor(self, "ones", (), {"shape": tuple(shape)})

    def evaluator(self) -> "Evaluator":
        return Evaluator(self)

    def num_nodes(self) -> int:
        return len(self._nodes)


Context = Graph


def run(fn, env=None):
    """Create a graph scope and call fn(ctx); returns fn's result."""
    return fn(Graph(env))


def _to_tensor(v, dtype=None, device=None):
    if isinstance(v, torch.Tensor):
        return v.to(device) if device is not None else v
    a = np.asarray(v)
    if a.dtype.kind in "iub":
        return torch.as_tensor(a, device=device)
    return torch.as_tensor(a, dtype=dtype or torch.float32, device=device)


class Evaluator:
    """Collects output nodes and feeds, evaluates them together
    (reference: scirs2-autograd/src/evaluation.rs)."""

    def __init__(self, graph: Graph):
        self.graph = graph
        self.targets: list[Tensor] = []
        self.feeds: dict = {}
        self.as_numpy = True

    def push(self, t: Tensor) -> "Evaluator":
        self.targets.append(t)
        return self

    def extend(self, ts) -> "Evaluator":
        self.targets.extend(ts)
        return self

    def feed(self, placeholder, value) -> "Evaluator":
        key = placeholder.attrs["name"] if isinstance(placeholder, Tensor) else placeholder
        self.feeds[key] = value
        return self

    def set_feeder(self, feeder: "Feeder") -> "Evaluator":
        self.feeds.update(feeder.values)
        return self

    def torch(self) -> "Evaluator":
        self.as_numpy = False
        return self

    def parallel(self, n_threads: int = 0) -> "Evaluator":
        """Evaluate independent nodes concurrently: the needed subgraph becomes a task graph on the
        native dataflow scheduler (a node starts when its inputs are ready). Tensor operations release
        the interpreter lock, so independent branches overlap (reference: scirs2-autograd/src/parallel,
        work-stealing graph evaluation)."""
        self.n_threads = n_threads
        self._parallel = True
        return self

    def run(self):
        from .ops import OPS

        memo: dict[int, torch.Tensor] = {}
        env = self.graph.env
        leaves: dict[int, torch.Tensor] = {}

        def ev(node: Tensor):
            if node.id in memo:
                return memo[node.id]
            op = node.op
            if op == "placeholder":
                name = node.attrs["name"]
                if name not in self.feeds:
                    raise KeyError(f"placeholder '{name}' was not fed")
                v = _to_tensor(self.feeds[name])
                if v.is_floating_point():
                    v = v.detach().requires_grad_(True)
                leaves[node.id] = v
            elif op == "variable":
                v = env.array(node.attrs["vid"]).detach()
                if v.is_floating_point():
                    v = v.requires_grad_(True)
                leaves[node.id] = v
            elif op == "grad":
                v = _eval_grad(node, ev)
            else:
                args = [ev(i) for i in node.inputs]
                v = OPS[op](*args, **node.attrs)
            for h in node.hooks:
                h(tuple(t.detach() for t in v) if isinstance(v, tuple) else v.detach())
            memo[node.id] = v
            return v

        order = self._topo_order()
        if getattr(self, "_parallel", False):
            self._run_parallel(ev, order)
        else:
            with torch.enable_grad():
                for n in order:  # dependencies first: ev never recurses deeply, whatever the graph depth
                    ev(n)
        with torch.enable_grad():
            outs = [ev(t) for t in self.targets]
        if self.as_numpy:
            return [o.detach().cpu().numpy() if isinstance(o, torch.Tensor) else o for o in outs]
        return [o.detach() if isinstance(o, torch.Tensor) else o for o in outs]

    @staticmethod
    def _deps(n: Tensor) -> list:
        if n.op == "grad":
            return list(n.attrs["ys"]) + list(n.attrs["xs"]) + list(n.attrs.get("gys") or [])
        return list(n.inputs)

    def _topo_order(self) -> list:
        """Every node the targets need, dependencies before dependents (iterative post-order DFS)."""
        order, seen, stack = [], set(), [(t, False) for t in reversed(self.targets)]
        while stack:
            n, done = stack.pop()
            if done:
                order.append(n)
                continue
            if n.id in seen:
                continue
            seen.add(n.id)
            stack.append((n, True))
            stack.extend((d, False) for d in reversed(self._deps(n)) if d.id not in seen)
        return order

    def _run_parallel(self, ev, order) -> None:
        from ..parallel.primitives import TaskGraph

        deps = self._deps
        tg = TaskGraph(getattr(self, "n_threads", 0))

        def task(n):
            def body(_):
                with torch.enable_grad():
                    ev(n)

            return body

        for n in order:
            tg.add_task(str(n.id), sorted({str(d.id) for d in deps(n)}), task(n))
        tg.execute()


def _eval_grad(node: Tensor, ev):
    ys = [ev(y) for y in node.attrs["ys"]]
    xs = [ev(x) for x in node.attrs["xs"]]
    gys = node.attrs.get("gys")
    gys = [ev(g) for g in gys] if gys is not None else [torch.ones_like(y) for y in ys]
    pairs = [(y, g) for y, g in zip(ys, gys) if y.requires_grad]
    if not pairs:
        return torch.zeros_like(xs[node.attrs["k"]])
    gs = torch.autograd.grad([p[0] for p in pairs], xs, [p[1] for p in pairs], create_graph=True, allow_unused=True)
    g = gs[node.attrs["k"]]
    return torch.zeros_like(xs[node.attrs["k"]]) if g is None else g


def grad(ys, xs, gys=None):
    """Symbolic gradients d(sum ys)/d xs (reference: tensor_ops/mod.rs:600,
    gradient.rs:20-116). Returns one node per x."""
    ys = list(ys) if isinstance(ys, (list, tuple)) else [ys]
    xs = list(xs) if isinstance(xs, (list, tuple)) else [xs]
    g = ys[0].graph
    return [Tensor(g, "grad", (), {"ys": ys, "xs": xs, "k": k, "gys": gys}) for k in range(len(xs))]


class Feeder:
    def __init__(self):
        self.values = {}

    def push(self, placeholder, value) -> "Feeder":
        key = placeholder.attrs["name"] if isinstance(placeholder, Tensor) else placeholder
        self.values[key] = value
        return self
