"""Graph rewriting and scheduling for the define-then-run graphs.

Rewrites (in place, on the nodes reachable from the given outputs):
  eliminate_common_subexpressions  nodes with the same op, the same
      (canonical) inputs and equal attributes are merged; inputs are rewired
      to the first occurrence
  fold_constants  a pure node whose inputs are all constants is evaluated
      once and becomes a constant
  simplify  algebraic identities: x*1, 1*x, x+0, 0+x, x-0, x/1, neg(neg x)
  fusion_groups  maximal chains of elementwise ops whose intermediate results
      have a single consumer (candidates for one fused kernel)

Scheduling / analysis:
  forward_schedule / reverse_schedule  topological orders (inputs first /
      outputs first)
  memory_optimal_schedule  greedy list schedule that, among the ready nodes,
      runs the one that frees the most bytes (ties: fewest new bytes)
  liveness / peak_memory / assign_memory_slots  live intervals of every value
      under a schedule, the peak of the live bytes, and a first-fit reuse of
      buffer slots between values whose intervals do not overlap
  level_decomposition / critical_path  nodes grouped by depth (independent
      within a level), and the longest path by a per-op cost

Reference parity: scirs2-autograd/src/optimization/{cse.rs,
constant_folding.rs, expression_simplification.rs, fusion/,
memory_optimization.rs} and scheduling/{topological.rs:12-330,
memory_planner.rs:13-380, parallel_schedule.rs:13-400}.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .graph import Tensor

_SOURCES = {"placeholder", "variable", "constant", "zeros", "ones"}
_IMPURE = {"placeholder", "variable", "grad", "random_normal", "random_uniform", "dropout", "bernoulli"}
_ELEMENTWISE = {"add", "sub", "mul", "div", "neg", "pow", "exp", "log", "sqrt", "square", "abs", "relu", "sigmoid",
                "tanh", "gelu", "softplus", "sin", "cos", "maximum", "minimum", "clip"}


def reachable(outputs) -> list[Tensor]:
    """Nodes reachable from `outputs`, inputs before consumers."""
    order, seen = [], set()
    stack = [(o, False) for o in reversed(list(outputs))]
    while stack:
        n, done = stack.pop()
        if done:
            order.append(n)
            continue
        if n.id in seen:
            continue
        seen.add(n.id)
        stack.append((n, True))
        for i in reversed(n.inputs):
            if i.id not in seen:
                stack.append((i, False))
    return order


def consumers(nodes) -> dict[int, list[Tensor]]:
    out = {n.id: [] for n in nodes}
    for n in nodes:
        for i in n.inputs:
            out.setdefault(i.id, []).append(n)
    return out


def _attr_key(attrs: dict):
    key = []
    for k in sorted(attrs):
        v = attrs[k]
        if isinstance(v, (torch.Tensor, np.ndarray)):
            return None  # array attributes: never merged
        try:
            hash(v)
            key.append((k, v))
        except TypeError:
            key.append((k, repr(v)))
    return tuple(key)


def eliminate_common_subexpressions(outputs) -> int:
    """Merge duplicate nodes; returns how many were removed from the
    reachable graph. `outputs` keep their identity (their inputs are
    rewired)."""
    canon: dict[int, Tensor] = {}
    table: dict = {}
    removed = 0
    for n in reachable(outputs):
        n.inputs = tuple(canon.get(i.id, i) for i in n.inputs)
        if n.op in _IMPURE:
            canon[n.id] = n
            continue
        ak = _attr_key(n.attrs)
        if ak is None:
            canon[n.id] = n
            continue
        key = (n.op, tuple(i.id for i in n.inputs), ak)
        first = table.get(key)
        if first is None:
            table[key] = n
            canon[n.id] = n
        else:
            canon[n.id] = first
            removed += 1
    for o in outputs:  # an output that duplicated an earlier node keeps its own identity
        if canon.get(o.id, o) is not o:
            f = canon[o.id]
            o.op, o.inputs, o.attrs = f.op, f.inputs, f.attrs
    return removed


def fold_constants(outputs) -> int:
    folded = 0
    for n in reachable(outputs):
        if n.op in _SOURCES or n.op in _IMPURE or n.op == "grad" or not n.inputs:
            continue
        if all(i.op == "constant" for i in n.inputs):
            value = n.graph.evaluator().push(n).run()[0]
            n.op, n.inputs, n.attrs = "constant", (), {"value": value}
            folded += 1
    return folded


def _is_const(n: Tensor, v: float) -> bool:
    if n.op != "constant":
        return False
    x = n.attrs.get("value")
    try:
        a = np.asarray(x.detach().cpu() if isinstance(x, torch.Tensor) else x)
        return a.size == 1 and float(a) == v
    except Exception:
        return False


def simplify(outputs) -> int:
    """Rewrite algebraic identities; a simplified node becomes an `identity`
    of the surviving operand. Returns the number of rewrites."""
    count = 0
    for n in reachable(outputs):
        keep = None
        if n.op == "mul" and len(n.inputs) == 2:
            a, b = n.inputs
            keep = a if _is_const(b, 1.0) else (b if _is_const(a, 1.0) else None)
        elif n.op == "add" and len(n.inputs) == 2:
            a, b = n.inputs
            keep = a if _is_const(b, 0.0) else (b if _is_const(a, 0.0) else None)
        elif n.op == "sub" and len(n.inputs) == 2 and _is_const(n.inputs[1], 0.0):
            keep = n.inputs[0]
        elif n.op == "div" and len(n.inputs) == 2 and _is_const(n.inputs[1], 1.0):
            keep = n.inputs[0]
        elif n.op == "neg" and n.inputs[0].op == "neg":
            keep = n.inputs[0].inputs[0]
        if keep is not None:
            n.op, n.inputs, n.attrs = "identity", (keep,), {}
            count += 1
    return count


def fusion_groups(outputs) -> list[list[Tensor]]:
    """Chains of elementwise nodes in which every node except the last has
    exactly one consumer, which is the next node of the chain."""
    nodes = reachable(outputs)
    cons = consumers(nodes)
    out_ids = {o.id for o in outputs}
    groups, used = [], set()
    for n in nodes:
        if n.op not in _ELEMENTWISE or n.id in used:
            continue
        chain = [n]
        cur = n
        while cur.id not in out_ids and len(cons.get(cur.id, [])) == 1 and cons[cur.id][0].op in _ELEMENTWISE:
            cur = cons[cur.id][0]
            chain.append(cur)
        if len(chain) > 1:
            groups.append(chain)
            used.update(x.id for x in chain)
    return groups


# ----------------------------------------------------------------- scheduling
@dataclass
class Schedule:
    order: list = field(default_factory=list)
    direction: str = "forward"

    def ids(self) -> list[int]:
        return [n.id for n in self.order]


def forward_schedule(outputs) -> Schedule:
    return Schedule(reachable(outputs), "forward")


def reverse_schedule(outputs) -> Schedule:
    return Schedule(list(reversed(reachable(outputs))), "reverse")


def validate_schedule(sched: Schedule) -> bool:
    pos = {n.id: k for k, n in enumerate(sched.order)}
    for n in sched.order:
        for i in n.inputs:
            if i.id in pos and (pos[i.id] > pos[n.id]) == (sched.direction == "forward"):
                return False
    return True


def _size(n: Tensor, sizes) -> int:
    if sizes is not None and n.id in sizes:
        return int(sizes[n.id])
    if n.shape_hint:
        return int(np.prod([max(1, int(d)) for d in n.shape_hint])) * 4
    return 4


def memory_optimal_schedule(outputs, sizes: dict | None = None) -> Schedule:
    nodes = reachable(outputs)
    cons = consumers(nodes)
    remaining = {n.id: len(cons.get(n.id, [])) for n in nodes}
    pending_inputs = {n.id: len({i.id for i in n.inputs}) for n in nodes}
    ready = [n for n in nodes if pending_inputs[n.id] == 0]
    out_ids = {o.id for o in outputs}
    order = []
    while ready:
        def score(n):
            freed = sum(_size(i, sizes) for i in {i.id: i for i in n.inputs}.values()
                        if remaining[i.id] == 1 and i.id not in out_ids)
            return (-freed, _size(n, sizes), n.id)

        ready.sort(key=score)
        n = ready.pop(0)
        order.append(n)
        for i in {i.id: i for i in n.inputs}.values():
            remaining[i.id] -= 1
        for c in {c.id: c for c in cons.get(n.id, [])}.values():
            pending_inputs[c.id] -= 1
            if pending_inputs[c.id] == 0:
                ready.append(c)
    return Schedule(order, "forward")


@dataclass
class LivenessInterval:
    node_id: int
    start: int
    end: int
    size: int

    def overlaps(self, other: "LivenessInterval") -> bool:
        return self.start <= other.end and other.start <= self.end


def liveness(sched: Schedule, outputs, sizes: dict | None = None) -> list[LivenessInterval]:
    pos = {n.id: k for k, n in enumerate(sched.order)}
    last = {n.id: pos[n.id] for n in sched.order}
    for n in sched.order:
        for i in n.inputs:
            last[i.id] = max(last[i.id], pos[n.id])
    end = len(sched.order) - 1
    for o in outputs:
        last[o.id] = end
    return [LivenessInterval(n.id, pos[n.id], last[n.id], _size(n, sizes)) for n in sched.order]


def peak_memory(intervals: list[LivenessInterval]) -> int:
    if not intervals:
        return 0
    n = max(iv.end for iv in intervals) + 2
    delta = [0] * n
    for iv in intervals:
        delta[iv.start] += iv.size
        delta[iv.end + 1] -= iv.size
    live = peak = 0
    for d in delta:
        live += d
        peak = max(peak, live)
    return peak


def assign_memory_slots(intervals: list[LivenessInterval]) -> dict[int, int]:
    """First-fit: each value gets the lowest slot whose previous occupant's
    interval ended before it starts (slots are reused, sizes not merged)."""
    slot_end: list[int] = []
    out = {}
    for iv in sorted(intervals, key=lambda v: (v.start, v.node_id)):
        for s, e in enumerate(slot_end):
            if e < iv.start:
                slot_end[s] = iv.end
                out[iv.node_id] = s
                break
        else:
            out[iv.node_id] = len(slot_end)
            slot_end.append(iv.end)
    return out


def level_decomposition(outputs) -> list[list[Tensor]]:
    depth = {}
    for n in reachable(outputs):
        depth[n.id] = 1 + max((depth[i.id] for i in n.inputs), default=-1)
    levels: dict[int, list] = {}
    for n in reachable(outputs):
        levels.setdefault(depth[n.id], []).append(n)
    return [levels[k] for k in sorted(levels)]


def critical_path(outputs, cost=None) -> tuple[list[Tensor], float]:
    """Longest path (sum of `cost(node)`, default 1 per non-source node)."""
    cost = cost or (lambda n: 0.0 if n.op in _SOURCES else 1.0)
    best, prev = {}, {}
    for n in reachable(outputs):
        c = cost(n)
        if n.inputs:
            p = max(n.inputs, key=lambda i: best[i.id])
            best[n.id], prev[n.id] = best[p.id] + c, p
        else:
            best[n.id], prev[n.id] = c, None
    end = max(outputs, key=lambda o: best[o.id])
    path, cur = [], end
    while cur is not None:
        path.append(cur)
        cur = prev[cur.id]
    return list(reversed(path)), best[end.id]
