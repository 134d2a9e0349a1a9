"""Static computation graphs for inference: a builder that records layers as
nodes, an optimizer (dead-node elimination and Linear -> ReLU fusion) and an
executor that runs the graph with a weight map.

The executor computes with torch tensors on the device of its weights; its
Linear and LayerNorm nodes go through `ops.functional`, so on CUDA bf16 they
run on the framework's GEMM (the fused Linear + ReLU node becomes one GEMM
with a ReLU epilogue pass) and LayerNorm kernels. `trace_sequential` builds a
graph and its weight map from a torch `nn.Sequential` of Linear / ReLU /
Sigmoid / Tanh / LayerNorm / Softmax / Flatten layers.

Kept identical to the reference so graphs and weight maps port directly: node
ids are allocated in build order; graph inputs are `Constant` nodes without
inputs; Linear weights are looked up as `linear_{id}_weight` ([out, in],
row-major) and `linear_{id}_bias`; LayerNorm scales as `layer_norm_{id}_gamma`
/ `layer_norm_{id}_beta` (optional); a fused Linear + ReLU node keeps the
Linear node's id (so its weight keys); BatchNorm nodes pass their input
through and Conv1d / Transpose nodes are not executable. Softmax here
normalises along the node's `dim` (default 1) of its output shape.

Reference parity: scirs2-neural/src/tracing/types.rs:15-230 (DType,
TensorSpec, OpAttr, OpType, OpNode, StaticGraph, TraceConfig),
graph_builder.rs:34-300 (GraphBuilder), executor.rs:32-460 (GraphExecutor,
optimize: dead-node elimination, operator fusion).
"""
from __future__ import annotations

import json
from collections import deque
from dataclasses import dataclass, field
from enum import Enum

import torch
import torch.nn as tnn


class DType(Enum):
    F16 = "f16"
    BF16 = "bf16"
    F32 = "f32"
    F64 = "f64"
    I32 = "i32"
    I64 = "i64"


@dataclass
class TensorSpec:
    shape: list
    dtype: DType = DType.F64

    def num_elements(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n


class OpType(Enum):
    LINEAR = "Linear"
    CONV1D = "Conv1d"
    RELU = "ReLU"
    SIGMOID = "Sigmoid"
    TANH = "Tanh"
    ADD = "Add"
    MUL = "Mul"
    RESHAPE = "Reshape"
    TRANSPOSE = "Transpose"
    SOFTMAX = "Softmax"
    LAYER_NORM = "LayerNorm"
    BATCH_NORM = "BatchNorm"
    FUSED_LINEAR_RELU = "FusedLinearReLU"
    CONSTANT = "Constant"


@dataclass
class OpNode:
    id: int
    op_type: OpType
    inputs: list
    attrs: dict
    output_spec: TensorSpec
    outputs: list = field(default_factory=list)
    name: str | None = None


@dataclass
class TraceConfig:
    optimize: bool = True
    fold_constants: bool = True


class StaticGraph:
    def __init__(self, inputs: list, outputs: list):
        self.inputs, self.outputs = list(inputs), list(outputs)
        self.nodes: list[OpNode] = []
        self.id_to_idx: dict[int, int] = {}
        self.input_node_ids: list[int] = []
        self.output_node_ids: list[int] = []

    def get_node(self, node_id: int) -> OpNode | None:
        i = self.id_to_idx.get(node_id)
        return self.nodes[i] if i is not None else None

    def num_nodes(self) -> int:
        return len(self.nodes)

    def to_json(self) -> str:
        def spec(s):
            return {"shape": list(s.shape), "dtype": s.dtype.value}

        return json.dumps({
            "inputs": [spec(s) for s in self.inputs], "outputs": [spec(s) for s in self.outputs],
            "input_node_ids": self.input_node_ids, "output_node_ids": self.output_node_ids,
            "nodes": [{"id": n.id, "op": n.op_type.value, "inputs": n.inputs, "outputs": n.outputs,
                       "attrs": n.attrs, "spec": spec(n.output_spec), "name": n.name} for n in self.nodes]})

    @staticmethod
    def from_json(text: str) -> "StaticGraph":
        d = json.loads(text)
        sp = lambda s: TensorSpec(list(s["shape"]), DType(s["dtype"]))  # noqa: E731
        g = StaticGraph([sp(s) for s in d["inputs"]], [sp(s) for s in d["outputs"]])
        for n in d["nodes"]:
            g.nodes.append(OpNode(n["id"], OpType(n["op"]), list(n["inputs"]), dict(n["attrs"]), sp(n["spec"]),
                                  list(n["outputs"]), n["name"]))
        g.id_to_idx = {n.id: i for i, n in enumerate(g.nodes)}
        g.input_node_ids, g.output_node_ids = list(d["input_node_ids"]), list(d["output_node_ids"])
        return g


@dataclass(frozen=True)
class GraphTensor:
    """Handle to a node's output while building."""

    id: int


class GraphBuilder:
    def __init__(self):
        self.nodes: list[OpNode] = []
        self._consumers: dict[int, list[int]] = {}
        self._next = 0

    def _spec(self, t: GraphTensor) -> TensorSpec:
        for n in self.nodes:
            if n.id == t.id:
                return n.output_spec
        raise ValueError(f"unknown tensor {t.id}")

    def _add(self, op: OpType, inputs: list, attrs: dict, spec: TensorSpec, prefix: str) -> GraphTensor:
        nid = self._next
        self._next += 1
        self.nodes.append(OpNode(nid, op, [t.id for t in inputs], attrs, spec, name=f"{prefix}_{nid}"))
        for t in inputs:
            self._consumers.setdefault(t.id, []).append(nid)
        return GraphTensor(nid)

    def input(self, spec: TensorSpec) -> GraphTensor:
        return self._add(OpType.CONSTANT, [], {}, spec, "input")

    def linear(self, x: GraphTensor, in_features: int, out_features: int) -> GraphTensor:
        shape = list(self._spec(x).shape) or [1, in_features]
        shape[-1] = out_features
        return self._add(OpType.LINEAR, [x], {"in_features": int(in_features), "out_features": int(out_features)},
                         TensorSpec(shape), "linear")

    def _unary(self, op, x, prefix):
        return self._add(op, [x], {}, TensorSpec(list(self._spec(x).shape)), prefix)

    def relu(self, x):
        return self._unary(OpType.RELU, x, "relu")

    def sigmoid(self, x):
        return self._unary(OpType.SIGMOID, x, "sigmoid")

    def tanh(self, x):
        return self._unary(OpType.TANH, x, "tanh")

    def add(self, a, b):
        return self._add(OpType.ADD, [a, b], {}, TensorSpec(list(self._spec(a).shape)), "add")

    def mul(self, a, b):
        return self._add(OpType.MUL, [a, b], {}, TensorSpec(list(self._spec(a).shape)), "mul")

    def reshape(self, x, new_shape: list):
        if TensorSpec(list(new_shape)).num_elements() != self._spec(x).num_elements():
            raise ValueError("reshape must keep the number of elements")
        return self._add(OpType.RESHAPE, [x], {"shape": [int(s) for s in new_shape]}, TensorSpec(list(new_shape)),
                         "reshape")

    def softmax(self, x, dim: int = 1):
        return self._add(OpType.SOFTMAX, [x], {"dim": int(dim)}, TensorSpec(list(self._spec(x).shape)), "softmax")

    def layer_norm(self, x, eps: float = 1e-5):
        return self._add(OpType.LAYER_NORM, [x], {"eps": float(eps)}, TensorSpec(list(self._spec(x).shape)),
                         "layer_norm")

    def build(self, outputs: list) -> StaticGraph:
        for n in self.nodes:
            n.outputs = list(self._consumers.get(n.id, []))
        ins = [n for n in self.nodes if n.op_type is OpType.CONSTANT and not n.inputs]
        by_id = {n.id: n for n in self.nodes}
        g = StaticGraph([n.output_spec for n in ins], [by_id[t.id].output_spec for t in outputs if t.id in by_id])
        g.nodes = list(self.nodes)
        g.id_to_idx = {n.id: i for i, n in enumerate(g.nodes)}
        g.input_node_ids = [n.id for n in ins]
        g.output_node_ids = [t.id for t in outputs]
        return g


def optimize(graph: StaticGraph) -> StaticGraph:
    """Dead-node elimination (keep what the outputs depend on), then Linear -> ReLU fusion where the
    Linear's only consumer is the ReLU (the fused node keeps the Linear's id; the ReLU's consumers
    and the graph outputs are rewired to it)."""
    live, q = set(graph.output_node_ids), deque(graph.output_node_ids)
    by_id = {n.id: n for n in graph.nodes}
    while q:
        nid = q.popleft()
        for p in by_id[nid].inputs:
            if p not in live:
                live.add(p)
                q.append(p)
    nodes = [OpNode(n.id, n.op_type, list(n.inputs), dict(n.attrs), n.output_spec,
                    [c for c in n.outputs if c in live], n.name) for n in graph.nodes if n.id in live]
    nodes_by_id = {n.id: n for n in nodes}
    consumers = {n.id: [m.id for m in nodes if n.id in m.inputs] for n in nodes}
    relu_to_lin = {}
    for n in nodes:
        if n.op_type is OpType.RELU and n.inputs:
            lin = nodes_by_id.get(n.inputs[0])
            if lin is not None and lin.op_type is OpType.LINEAR and consumers[lin.id] == [n.id] \
                    and lin.id not in graph.output_node_ids:
                relu_to_lin[n.id] = lin.id
    out = []
    for n in nodes:
        if n.id in relu_to_lin:
            continue
        if n.id in relu_to_lin.values():
            relu = next(r for r, lid in relu_to_lin.items() if lid == n.id)
            n = OpNode(n.id, OpType.FUSED_LINEAR_RELU, n.inputs, n.attrs, nodes_by_id[relu].output_spec,
                       list(nodes_by_id[relu].outputs), f"fused_linear_relu_{n.id}")
        n.inputs = [relu_to_lin.get(i, i) for i in n.inputs]
        out.append(n)
    g = StaticGraph(graph.inputs, graph.outputs)
    g.nodes = out
    g.id_to_idx = {n.id: i for i, n in enumerate(out)}
    g.input_node_ids = list(graph.input_node_ids)
    g.output_node_ids = [relu_to_lin.get(i, i) for i in graph.output_node_ids]
    return g


class GraphExecutor:
    def __init__(self, graph: StaticGraph, weight_map: dict, device=None, dtype=torch.float64):
        self.graph = graph
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.weights = {k: torch.as_tensor(v, dtype=dtype, device=self.device) for k, v in weight_map.items()}

    def _linear(self, node, x, relu):
        from ..ops import functional as OF

        i, o = node.attrs["in_features"], node.attrs["out_features"]
        w, b = self.weights.get(f"linear_{node.id}_weight"), self.weights.get(f"linear_{node.id}_bias")
        if w is None or b is None:
            raise ValueError(f"missing weight 'linear_{node.id}_weight' or bias 'linear_{node.id}_bias'")
        if w.numel() != o * i:
            raise ValueError(f"weight shape mismatch: expected {o}x{i}, got {w.numel()}")
        if x.numel() % i:
            raise ValueError(f"input length {x.numel()} not divisible by in_features {i}")
        y = OF.linear(x.reshape(-1, i), w.reshape(o, i).t(), b.reshape(o))
        return torch.relu(y) if relu else y

    def run(self, inputs: list) -> list:
        g = self.graph
        if len(inputs) != len(g.input_node_ids):
            raise ValueError(f"expected {len(g.input_node_ids)} inputs, got {len(inputs)}")
        cache = {nid: torch.as_tensor(x, dtype=self.dtype, device=self.device).reshape(
            g.get_node(nid).output_spec.shape) for x, nid in zip(inputs, g.input_node_ids)}
        for n in g.nodes:
            if n.op_type is OpType.CONSTANT:
                cache.setdefault(n.id, torch.zeros(n.output_spec.shape, dtype=self.dtype, device=self.device))
                continue
            x = [cache[i] for i in n.inputs]
            t = n.op_type
            if t in (OpType.LINEAR, OpType.FUSED_LINEAR_RELU):
                y = self._linear(n, x[0], t is OpType.FUSED_LINEAR_RELU)
            elif t is OpType.RELU:
                y = torch.relu(x[0])
            elif t is OpType.SIGMOID:
                y = torch.sigmoid(x[0])
            elif t is OpType.TANH:
                y = torch.tanh(x[0])
            elif t is OpType.ADD:
                y = x[0] + x[1]
            elif t is OpType.MUL:
                y = x[0] * x[1]
            elif t is OpType.RESHAPE:
                y = x[0].reshape(n.output_spec.shape)
            elif t is OpType.SOFTMAX:
                shp = n.output_spec.shape
                dim = n.attrs.get("dim", 1)
                xs = x[0].reshape(shp)
                y = torch.softmax(xs, dim=dim if dim < len(shp) else -1)
            elif t is OpType.LAYER_NORM:
                from ..ops import functional as OF

                d = n.output_spec.shape[-1]
                gmm = self.weights.get(f"layer_norm_{n.id}_gamma", torch.ones(d, dtype=self.dtype, device=self.device))
                bta = self.weights.get(f"layer_norm_{n.id}_beta", torch.zeros(d, dtype=self.dtype, device=self.device))
                y = OF.layer_norm(x[0].reshape(-1, d), gmm, bta, n.attrs.get("eps", 1e-5))
            elif t is OpType.BATCH_NORM:
                y = x[0]
            else:
                raise NotImplementedError(f"{t.value} is not executable")
            cache[n.id] = y.reshape(n.output_spec.shape)
        missing = [o for o in g.output_node_ids if o not in cache]
        if missing:
            raise ValueError(f"output nodes {missing} not computed")
        return [cache[o] for o in g.output_node_ids]


def trace_sequential(model: tnn.Sequential, input_shape: list, config: TraceConfig | None = None):
    """Graph and weight map of a torch nn.Sequential (Linear, ReLU, Sigmoid, Tanh, LayerNorm over the
    last dimension, Softmax, Flatten); `config.optimize` runs `optimize`."""
    config = config or TraceConfig()
    gb = GraphBuilder()
    x = gb.input(TensorSpec(list(input_shape)))
    weights = {}
    for m in model:
        shp = list(gb._spec(x).shape)
        if isinstance(m, tnn.Linear):
            x = gb.linear(x, m.in_features, m.out_features)
            weights[f"linear_{x.id}_weight"] = m.weight.detach().double().reshape(-1).tolist()
            bias = m.bias.detach() if m.bias is not None else torch.zeros(m.out_features)
            weights[f"linear_{x.id}_bias"] = bias.double().tolist()
        elif isinstance(m, tnn.ReLU):
            x = gb.relu(x)
        elif isinstance(m, tnn.Sigmoid):
            x = gb.sigmoid(x)
        elif isinstance(m, tnn.Tanh):
            x = gb.tanh(x)
        elif isinstance(m, tnn.Flatten):
            x = gb.reshape(x, shp[:m.start_dim] + [int(torch.tensor(shp[m.start_dim:]).prod())])
        elif isinstance(m, tnn.LayerNorm):
            if len(m.normalized_shape) != 1:
                raise ValueError("LayerNorm over the last dimension only")
            x = gb.layer_norm(x, m.eps)
            if m.weight is not None:
                weights[f"layer_norm_{x.id}_gamma"] = m.weight.detach().double().tolist()
                weights[f"layer_norm_{x.id}_beta"] = m.bias.detach().double().tolist()
        elif isinstance(m, tnn.Softmax):
            x = gb.softmax(x, m.dim if m.dim is not None and m.dim >= 0 else len(shp) - 1)
        else:
            raise ValueError(f"cannot trace {type(m).__name__}")
    g = gb.build([x])
    return (optimize(g) if config.optimize else g), weights
