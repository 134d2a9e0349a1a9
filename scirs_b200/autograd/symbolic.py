"""Symbolic expressions: build, differentiate, simplify, evaluate; and a
symbolic tape (recorded scalar program with reverse-mode gradients).

Reference parity: scirs2-autograd/src/symbolic/{expression.rs,
rules.rs (chain / product / quotient rules), simplify.rs,
symbolic_tape.rs}.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class SymExpr:
    op: str                 # const | var | add | mul | pow | neg | exp | log | sin | cos | div
    args: tuple = ()
    value: float = 0.0      # const value / pow exponent
    name: str = ""

    # ---------------------------------------------------------- builders
    @staticmethod
    def constant(v: float) -> "SymExpr":
        return SymExpr("const", value=float(v))

    @staticmethod
    def variable(name: str) -> "SymExpr":
        return SymExpr("var", name=name)

    def __add__(self, o):
        return SymExpr("add", (self, _e(o)))

    __radd__ = __add__

    def __mul__(self, o):
        return SymExpr("mul", (self, _e(o)))

    __rmul__ = __mul__

    def __sub__(self, o):
        return self + (-_e(o))

    def __rsub__(self, o):
        return _e(o) + (-self)

    def __truediv__(self, o):
        return SymExpr("div", (self, _e(o)))

    def __neg__(self):
        return SymExpr("neg", (self,))

    def __pow__(self, p: float):
        return SymExpr("pow", (self,), value=float(p))

    # ---------------------------------------------------------- calculus
    def differentiate(self, var: str) -> "SymExpr":
        o, a = self.op, self.args
        if o == "const":
            return C(0)
        if o == "var":
            return C(1.0 if self.name == var else 0.0)
        if o == "add":
            return a[0].differentiate(var) + a[1].differentiate(var)
        if o == "mul":  # product rule
            return a[0].differentiate(var) * a[1] + a[0] * a[1].differentiate(var)
        if o == "div":  # quotient rule
            return (a[0].differentiate(var) * a[1] - a[0] * a[1].differentiate(var)) / (a[1] ** 2)
        if o == "neg":
            return -a[0].differentiate(var)
        if o == "pow":  # chain rule
            return C(self.value) * (a[0] ** (self.value - 1)) * a[0].differentiate(var)
        if o == "exp":
            return self * a[0].differentiate(var)
        if o == "log":
            return a[0].differentiate(var) / a[0]
        if o == "sin":
            return cos(a[0]) * a[0].differentiate(var)
        if o == "cos":
            return -(sin(a[0]) * a[0].differentiate(var))
        raise ValueError(o)

    def simplify(self) -> "SymExpr":
        return simplify_expr(self)

    def evaluate(self, vars: dict) -> float:
        o, a = self.op, self.args
        if o == "const":
            return self.value
        if o == "var":
            if self.name not in vars:
                raise KeyError(f"unbound variable {self.name}")
            return float(vars[self.name])
        x = [e.evaluate(vars) for e in a]
        return {"add": lambda: x[0] + x[1], "mul": lambda: x[0] * x[1], "div": lambda: x[0] / x[1],
                "neg": lambda: -x[0], "pow": lambda: x[0] ** self.value, "exp": lambda: math.exp(x[0]),
                "log": lambda: math.log(x[0]), "sin": lambda: math.sin(x[0]), "cos": lambda: math.cos(x[0])}[o]()

    def __str__(self):
        o, a = self.op, self.args
        if o == "const":
            return f"{self.value:g}"
        if o == "var":
            return self.name
        if o in ("add", "mul", "div"):
            return f"({a[0]} {dict(add='+', mul='*', div='/')[o]} {a[1]})"
        if o == "neg":
            return f"-{a[0]}"
        if o == "pow":
            return f"{a[0]}^{self.value:g}"
        return f"{o}({a[0]})"


def C(v):
    return SymExpr.constant(v)


def _e(x):
    return x if isinstance(x, SymExpr) else C(x)


def exp(x):
    return SymExpr("exp", (_e(x),))


def log(x):
    return SymExpr("log", (_e(x),))


def sin(x):
    return SymExpr("sin", (_e(x),))


def cos(x):
    return SymExpr("cos", (_e(x),))


def _c(e: SymExpr, v=None) -> bool:
    return e.op == "const" and (v is None or e.value == v)


def simplify_expr(e: SymExpr) -> SymExpr:
    """Bottom-up: fold constant sub-expressions, x+0, x*1, x*0, x^1, x^0,
    x/1, --x."""
    if e.op in ("const", "var"):
        return e
    a = tuple(simplify_expr(x) for x in e.args)
    e = SymExpr(e.op, a, e.value, e.name)
    if all(_c(x) for x in a):
        return C(e.evaluate({}))
    o = e.op
    if o == "add":
        if _c(a[0], 0):
            return a[1]
        if _c(a[1], 0):
            return a[0]
    if o == "mul":
        if _c(a[0], 0) or _c(a[1], 0):
            return C(0)
        if _c(a[0], 1):
            return a[1]
        if _c(a[1], 1):
            return a[0]
    if o == "div" and _c(a[1], 1):
        return a[0]
    if o == "pow":
        if e.value == 1:
            return a[0]
        if e.value == 0:
            return C(1)
    if o == "neg" and a[0].op == "neg":
        return a[0].args[0]
    return e


class ExprBuilder:
    def __init__(self, e: SymExpr):
        self.e = e

    @classmethod
    def var(cls, name):
        return cls(SymExpr.variable(name))

    @classmethod
    def constant(cls, v):
        return cls(C(v))

    def add(self, o):
        return ExprBuilder(self.e + _e(o.e if isinstance(o, ExprBuilder) else o))

    def mul(self, o):
        return ExprBuilder(self.e * _e(o.e if isinstance(o, ExprBuilder) else o))

    def pow(self, p):
        return ExprBuilder(self.e ** p)

    def build(self) -> SymExpr:
        return self.e


class SymbolicTape:
    """A recorded scalar program: each op appends a node; `forward` evaluates
    it, `gradient` runs reverse mode over the tape."""

    def __init__(self):
        self.nodes: list[tuple] = []  # (op, a, b, value/name)

    def _push(self, op, a=-1, b=-1, extra=None) -> int:
        self.nodes.append((op, a, b, extra))
        return len(self.nodes) - 1

    def input(self, name: str) -> int:
        return self._push("input", extra=name)

    def constant(self, v: float) -> int:
        return self._push("const", extra=float(v))

    def add(self, a, b):
        return self._push("add", a, b)

    def sub(self, a, b):
        return self._push("sub", a, b)

    def mul(self, a, b):
        return self._push("mul", a, b)

    def div(self, a, b):
        return self._push("div", a, b)

    def exp(self, a):
        return self._push("exp", a)

    def log(self, a):
        return self._push("log", a)

    def forward(self, inputs: dict) -> list[float]:
        v = []
        for op, a, b, x in self.nodes:
            v.append({"input": lambda: float(inputs[x]), "const": lambda: x, "add": lambda: v[a] + v[b],
                      "sub": lambda: v[a] - v[b], "mul": lambda: v[a] * v[b], "div": lambda: v[a] / v[b],
                      "exp": lambda: math.exp(v[a]), "log": lambda: math.log(v[a])}[op]())
        return v

    def gradient(self, inputs: dict, output: int) -> dict:
        v = self.forward(inputs)
        g = [0.0] * len(v)
        g[output] = 1.0
        for i in range(output, -1, -1):
            op, a, b, _ = self.nodes[i]
            gi = g[i]
            if op == "add":
                g[a] += gi
                g[b] += gi
            elif op == "sub":
                g[a] += gi
                g[b] -= gi
            elif op == "mul":
                g[a] += gi * v[b]
                g[b] += gi * v[a]
            elif op == "div":
                g[a] += gi / v[b]
                g[b] -= gi * v[a] / v[b] ** 2
            elif op == "exp":
                g[a] += gi * v[i]
            elif op == "log":
                g[a] += gi / v[a]
        return {x: g[i] for i, (op, _, _, x) in enumerate(self.nodes) if op == "input"}
