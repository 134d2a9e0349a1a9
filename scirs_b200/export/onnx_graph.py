"""ONNX export of autograd graphs, a fluent ONNX graph builder and tensor
conversions.

`export_graph(outputs, feeds)` walks the nodes of a graph built with the
define-then-run API (:mod:`scirs_b200.autograd`) that the outputs depend on
and emits one ONNX node (or a short fixed pattern) per graph node:
placeholders become graph inputs, variables and constants become
initializers (their current values), every other node maps to the ONNX
operator of the same math. Shapes come from evaluating the graph once on
`feeds`. The result is an :class:`OnnxModel` (protobuf bytes via
``to_bytes`` / ``save``, JSON via ``to_json``), and ``run_graph`` executes it
so an export can be checked against the graph's own evaluation.

`OnnxGraphBuilder` assembles a graph by hand (inputs, outputs,
initializers, typed helpers for the common operators, validation on
``build``). `tensor_to_onnx` / `onnx_to_tensor` convert between torch
tensors and ONNX tensors.

Reference parity: scirs2-autograd/src/onnx/builder.rs:47-520
(OnnxGraphBuilder with add_matmul / add_gemm / add_relu / ... / build),
convert.rs:29-200 (array <-> OnnxTensor), io.rs:34-120 (JSON export /
import). The wire format and graph IR are shared with the layer-model
exporter (scirs_b200/export/onnx.py).
"""
from __future__ import annotations

import torch

from .onnx import FLOAT, INT64, OnnxGraph, OnnxModel, OnnxNode, OnnxTensor, OnnxValueInfo, run_graph


# ----------------------------------------------------------------- tensors
def tensor_to_onnx(name: str, t: torch.Tensor) -> OnnxTensor:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8, torch.bool):
        return OnnxTensor(name, list(t.shape), t.long().reshape(-1).tolist(), INT64)
    return OnnxTensor(name, list(t.shape), t.float().reshape(-1).tolist(), FLOAT)


def onnx_to_tensor(t: OnnxTensor) -> torch.Tensor:
    return t.to_torch()


def _i64(name: str, values) -> OnnxTensor:
    vals = [int(v) for v in (values if isinstance(values, (list, tuple)) else [values])]
    return OnnxTensor(name, [len(vals)], vals, INT64)


# ----------------------------------------------------------------- builder
class OnnxGraphBuilder:
    """Fluent construction of an ONNX graph; `build()` checks that every
    node input is a graph input, an initializer or an earlier node's output,
    and that every graph output is produced."""

    def __init__(self, name: str):
        self.g = OnnxGraph(name)
        self.doc = ""

    def doc_string(self, doc: str) -> "OnnxGraphBuilder":
        self.doc = doc
        return self

    def add_input(self, name: str, dims, elem_type: int = FLOAT) -> "OnnxGraphBuilder":
        self.g.inputs.append(OnnxValueInfo(name, elem_type, list(dims)))
        return self

    def add_output(self, name: str, dims, elem_type: int = FLOAT) -> "OnnxGraphBuilder":
        self.g.outputs.append(OnnxValueInfo(name, elem_type, list(dims)))
        return self

    def add_initializer(self, tensor: OnnxTensor) -> "OnnxGraphBuilder":
        self.g.initializers.append(tensor)
        return self

    def add_node(self, node: OnnxNode) -> "OnnxGraphBuilder":
        self.g.nodes.append(node)
        return self

    def _op(self, op, name, ins, out, **attrs):
        return self.add_node(OnnxNode(op, name, list(ins), [out], dict(attrs)))

    def add_matmul(self, name, a, b, out):
        return self._op("MatMul", name, [a, b], out)

    def add_gemm(self, name, a, b, c, out, trans_a=0, trans_b=0, alpha=1.0, beta=1.0):
        return self._op("Gemm", name, [a, b] + ([c] if c else []), out, transA=trans_a, transB=trans_b,
                        alpha=float(alpha), beta=float(beta))

    def add_relu(self, name, x, out):
        return self._op("Relu", name, [x], out)

    def add_sigmoid(self, name, x, out):
        return self._op("Sigmoid", name, [x], out)

    def add_tanh(self, name, x, out):
        return self._op("Tanh", name, [x], out)

    def add_softmax(self, name, x, out, axis=-1):
        return self._op("Softmax", name, [x], out, axis=int(axis))

    def add_add(self, name, a, b, out):
        return self._op("Add", name, [a, b], out)

    def add_sub(self, name, a, b, out):
        return self._op("Sub", name, [a, b], out)

    def add_mul(self, name, a, b, out):
        return self._op("Mul", name, [a, b], out)

    def add_div(self, name, a, b, out):
        return self._op("Div", name, [a, b], out)

    def add_conv(self, name, x, w, out, kernel_shape, strides=(1, 1), pads=(0, 0, 0, 0), bias=None):
        return self._op("Conv", name, [x, w] + ([bias] if bias else []), out, kernel_shape=list(kernel_shape),
                        strides=list(strides), pads=list(pads))

    def add_max_pool(self, name, x, out, kernel_shape, strides):
        return self._op("MaxPool", name, [x], out, kernel_shape=list(kernel_shape), strides=list(strides))

    def add_average_pool(self, name, x, out, kernel_shape, strides):
        return self._op("AveragePool", name, [x], out, kernel_shape=list(kernel_shape), strides=list(strides))

    def add_global_average_pool(self, name, x, out):
        return self._op("GlobalAveragePool", name, [x], out)

    def add_batch_norm(self, name, x, scale, bias, mean, var, out, epsilon=1e-5):
        return self._op("BatchNormalization", name, [x, scale, bias, mean, var], out, epsilon=float(epsilon))

    def add_reshape(self, name, x, shape_name, out):
        return self._op("Reshape", name, [x, shape_name], out)

    def add_flatten(self, name, x, out, axis=1):
        return self._op("Flatten", name, [x], out, axis=int(axis))

    def add_transpose(self, name, x, out, perm):
        return self._op("Transpose", name, [x], out, perm=[int(p) for p in perm])

    def add_concat(self, name, inputs, out, axis):
        return self._op("Concat", name, list(inputs), out, axis=int(axis))

    def add_reduce_mean(self, name, x, out, axes_name=None, keepdims=0):
        return self._op("ReduceMean", name, [x] + ([axes_name] if axes_name else []), out, keepdims=int(keepdims))

    def add_reduce_sum(self, name, x, out, axes_name=None, keepdims=0):
        return self._op("ReduceSum", name, [x] + ([axes_name] if axes_name else []), out, keepdims=int(keepdims))

    def add_dropout(self, name, x, out):
        return self._op("Identity", name, [x], out)

    def add_leaky_relu(self, name, x, out, alpha=0.01):
        return self._op("LeakyRelu", name, [x], out, alpha=float(alpha))

    def add_clip(self, name, x, out, lo_name, hi_name):
        return self._op("Clip", name, [x, lo_name, hi_name], out)

    def add_identity(self, name, x, out):
        return self._op("Identity", name, [x], out)

    def build(self) -> OnnxGraph:
        known = {v.name for v in self.g.inputs} | {t.name for t in self.g.initializers}
        for n in self.g.nodes:
            for i in n.inputs:
                if i and i not in known:
                    raise ValueError(f"node {n.name} ({n.op_type}) reads undefined value '{i}'")
            known.update(n.outputs)
        for o in self.g.outputs:
            if o.name not in known:
                raise ValueError(f"graph output '{o.name}' is not produced by any node")
        return self.g

    def model(self) -> OnnxModel:
        return OnnxModel(self.build())


# ----------------------------------------------------------- graph export
_UNARY = {"exp": "Exp", "log": "Log", "sqrt": "Sqrt", "abs": "Abs", "sin": "Sin", "cos": "Cos", "tanh": "Tanh",
          "sigmoid": "Sigmoid", "relu": "Relu", "neg": "Neg", "identity": "Identity", "stop_gradient": "Identity",
          "softplus": "Softplus", "erf": "Erf", "floor": "Floor", "ceil": "Ceil", "sign": "Sign",
          "reciprocal": "Reciprocal", "tan": "Tan", "asin": "Asin", "acos": "Acos", "atan": "Atan",
          "sinh": "Sinh", "cosh": "Cosh", "round": "Round", "selu": "Selu", "softsign": "Softsign",
          "hard_sigmoid": "HardSigmoid", "hard_swish": "HardSwish", "mish": "Mish"}
_BINARY = {"add": "Add", "sub": "Sub", "mul": "Mul", "div": "Div", "matmul": "MatMul", "batch_matmul": "MatMul",
           "maximum": "Max", "minimum": "Min", "pow_tensor": "Pow", "bias_add": "Add"}


class _Emitter:
    def __init__(self, name, env):
        self.b = OnnxGraphBuilder(name)
        self.env = env
        self.names = {}
        self.k = 0

    def fresh(self, base):
        self.k += 1
        return f"{base}_{self.k}"

    def const(self, value, base="const"):
        name = self.fresh(base)
        self.b.add_initializer(tensor_to_onnx(name, torch.as_tensor(value)))
        return name


def export_graph(outputs, feeds: dict, name: str = "autograd_graph", opset: int = 20) -> OnnxModel:
    """Export the sub-graph that `outputs` (autograd graph nodes) depend on.
    `feeds` maps placeholder names to sample values (used for shapes and to
    fold node attributes); variables are read from the graph's
    VariableEnvironment and stored as initializers."""
    from ..autograd.graph import Tensor

    outputs = list(outputs) if isinstance(outputs, (list, tuple)) else [outputs]
    graph = outputs[0].graph
    # evaluate once for the output shapes
    ev = graph.evaluator().torch()
    for k, v in feeds.items():
        ev.feed(k, v)
    values = ev.extend(outputs).run()

    order, seen = [], set()
    stack: list[tuple[Tensor, bool]] = [(o, False) for o in reversed(outputs)]
    while stack:  # iterative post-order: inputs before their users, any graph depth
        n, done = stack.pop()
        if done:
            order.append(n)
            continue
        if n.id in seen:
            continue
        seen.add(n.id)
        if n.op == "grad":
            raise NotImplementedError("gradient nodes are not exported; export the forward graph")
        stack.append((n, True))
        stack.extend((i, False) for i in reversed(n.inputs) if i.id not in seen)

    em = _Emitter(name, graph.env)
    b = em.b
    for n in order:
        out = f"n{n.id}" if n.name is None else f"{n.name}_{n.id}"
        ins = [em.names[i.id] for i in n.inputs]
        a = n.attrs
        op = n.op
        if op == "placeholder":
            v = torch.as_tensor(feeds[a["name"]])
            b.add_input(a["name"], list(v.shape), INT64 if not v.is_floating_point() else FLOAT)
            em.names[n.id] = a["name"]
            continue
        if op == "variable":
            val = graph.env.array(a["vid"])
            b.add_initializer(tensor_to_onnx(out, val))
            em.names[n.id] = out
            continue
        if op == "constant":
            b.add_initializer(tensor_to_onnx(out, torch.as_tensor(a["value"])))
            em.names[n.id] = out
            continue
        if op in ("zeros", "ones"):
            b.add_initializer(tensor_to_onnx(out, (torch.zeros if op == "zeros" else torch.ones)(a["shape"])))
            em.names[n.id] = out
            continue
        if op in _UNARY:
            b._op(_UNARY[op], out, ins, out)
        elif op in _BINARY:
            b._op(_BINARY[op], out, ins, out)
        elif op == "square":
            b._op("Mul", out, [ins[0], ins[0]], out)
        elif op == "pow":
            b._op("Pow", out, [ins[0], em.const(float(a["p"]), "exponent")], out)
        elif op in ("softmax", "log_softmax"):
            b._op("Softmax" if op == "softmax" else "LogSoftmax", out, ins, out, axis=int(a["axis"]))
        elif op == "gelu":
            b._op("Gelu", out, ins, out, approximate="tanh")
        elif op in ("swish", "silu"):
            s = em.fresh("sig")
            b._op("Sigmoid", s, ins, s)
            b._op("Mul", out, [ins[0], s], out)
        elif op in ("leaky_relu", "elu"):
            b._op("LeakyRelu" if op == "leaky_relu" else "Elu", out, ins, out, alpha=float(a["alpha"]))
        elif op in ("reduce_sum", "reduce_mean", "reduce_max", "reduce_min", "reduce_prod"):
            onnx_op = {"reduce_sum": "ReduceSum", "reduce_mean": "ReduceMean", "reduce_max": "ReduceMax",
                       "reduce_min": "ReduceMin", "reduce_prod": "ReduceProd"}[op]
            axes = a["axes"]
            extra = []
            if axes is not None:
                extra = [em.const(torch.tensor(list(axes) if isinstance(axes, (list, tuple)) else [axes]), "axes")]
            b._op(onnx_op, out, ins + extra, out, keepdims=int(bool(a["keep_dims"])) if axes is not None else 0)
        elif op == "reshape":
            b._op("Reshape", out, [ins[0], em.const(torch.tensor(list(a["shape"])), "shape")], out)
        elif op == "transpose":
            perm = a["perm"] if a["perm"] is not None else [1, 0]
            b._op("Transpose", out, ins, out, perm=list(perm))
        elif op == "concat":
            b._op("Concat", out, ins, out, axis=int(a["axis"]))
        elif op == "expand_dims":
            b._op("Unsqueeze", out, [ins[0], em.const(torch.tensor([a["axis"]]), "axes")], out)
        elif op == "squeeze":
            b._op("Squeeze", out, [ins[0], em.const(torch.tensor([a["axis"]]), "axes")], out)
        elif op == "clip":
            b._op("Clip", out, [ins[0], em.const(float(a["lo"]), "lo"), em.const(float(a["hi"]), "hi")], out)
        elif op == "where":
            c = em.fresh("cond")
            b._op("Cast", c, [ins[0]], c, to=9)  # BOOL
            b._op("Where", out, [c, ins[1], ins[2]], out)
        elif op == "conv2d":
            w = n.inputs[1]
            wshape = list(values_of(graph, w, feeds).shape)
            s, p = a["stride"], a["padding"]
            s = [s, s] if isinstance(s, int) else list(s)
            p = [p, p] if isinstance(p, int) else list(p)
            b._op("Conv", out, ins, out, kernel_shape=wshape[2:], strides=s, pads=[p[0], p[1], p[0], p[1]])
        elif op in ("max_pool2d", "avg_pool2d"):
            k, s = a["size"], a["stride"]
            b._op("MaxPool" if op == "max_pool2d" else "AveragePool", out, ins, out, kernel_shape=[k, k],
                  strides=[s, s])
        elif op == "layer_norm":
            b._op("LayerNormalization", out, ins, out, axis=-1, epsilon=float(a["eps"]))
        elif op == "linear":
            mm = em.fresh("mm")
            b._op("MatMul", mm, ins[:2], mm)
            b._op("Add", out, [mm, ins[2]], out)
        elif op == "getitem" and isinstance(a["idx"], int):
            b._op("Gather", out, [ins[0], em.const(torch.tensor(a["idx"]), "index")], out, axis=0)
        else:
            raise NotImplementedError(f"ONNX export of graph op '{op}'")
        em.names[n.id] = out

    for o, v in zip(outputs, values):
        b.add_output(em.names[o.id], list(torch.as_tensor(v).shape))
    m = OnnxModel(b.build())
    m.opset = opset
    return m


def values_of(graph, node, feeds):
    ev = graph.evaluator().torch()
    for k, v in feeds.items():
        ev.feed(k, v)
    return ev.push(node).run()[0]


def run_onnx(model: OnnxModel, feeds: dict) -> list:
    """Execute an exported model; returns the graph outputs in order."""
    env = run_graph(model.graph, {k: torch.as_tensor(v) for k, v in feeds.items()})
    return [env[o.name] for o in model.graph.outputs]
