"""Model-graph IR: typed operator nodes, slot-to-slot edges and tensor shapes,
with JSON export / import, an ONNX-style JSON envelope, validation, a builder,
and capture of a PyTorch module's graph (torch.fx trace + shape propagation).

JSON layout (the reference's): `{"metadata": {...}, "nodes": [...], "edges":
[...]}`; each node carries `node_type` (input, output, dense, conv2_d,
depthwise_conv2_d, batch_norm, layer_norm, activation, max_pool2_d,
avg_pool2_d, global_avg_pool, dropout, reshape, flatten, add, concat,
attention, embedding, softmax, custom), `name`, `attrs` where the operator has
attributes, and `output_shape` (`shape` for input / output nodes) as
`{"dims": [int | null], "dtype": "f32" | "f64" | "f16" | "i32" | "i64" | "bool"}`;
an edge is `{"from_node", "from_slot", "to_node", "to_slot"}`.

`total_parameters()` counts the parameters the attributes imply (dense
in*out (+out), convolution out*in/groups*kh*kw (+out), affine norms 2*C,
embedding n*d, attention 4*d*d (+4*d)); the reference multiplies output sizes
by weight-tensor counts instead, which is not a parameter count.

Reference parity: scirs2-neural/src/serialization/model_graph.rs:33-1400
(TensorDtype, TensorShape, attribute structs, GraphNode, GraphEdge,
GraphMetadata, ModelGraph add / validate / export_to_json / import_from_json /
save / load / export_onnx_like, ModelGraphBuilder).
"""
from __future__ import annotations

import dataclasses
import json
import operator
from pathlib import Path

import torch
import torch.nn as nn

GRAPH_FORMAT_VERSION = "1.0"

_ONNX_ELEM = {"f32": 1, "i32": 6, "i64": 7, "bool": 9, "f16": 10, "f64": 11}
_TORCH_DT = {torch.float32: "f32", torch.float64: "f64", torch.float16: "f16", torch.bfloat16: "f16",
             torch.int32: "i32", torch.int64: "i64", torch.bool: "bool"}
_ONNX_OP = {"input": "Input", "output": "Output", "dense": "Gemm", "conv2_d": "Conv", "depthwise_conv2_d": "Conv",
            "batch_norm": "BatchNormalization", "layer_norm": "LayerNormalization", "max_pool2_d": "MaxPool",
            "avg_pool2_d": "AveragePool", "global_avg_pool": "GlobalAveragePool", "dropout": "Dropout",
            "reshape": "Reshape", "flatten": "Flatten", "add": "Add", "concat": "Concat",
            "attention": "MultiHeadAttention", "embedding": "Gather", "softmax": "Softmax"}
_ACT_OP = {"relu": "Relu", "sigmoid": "Sigmoid", "tanh": "Tanh", "gelu": "Gelu", "leaky_relu": "LeakyRelu",
           "elu": "Elu", "swish": "Swish", "silu": "Swish"}
NODE_TYPES = set(_ONNX_OP) | {"activation", "custom"}


class GraphError(ValueError):
    pass


@dataclasses.dataclass
class TensorShape:
    dims: list
    dtype: str = "f32"

    @classmethod
    def with_batch_dim(cls, spatial: list, dtype: str = "f32") -> "TensorShape":
        return cls([None] + list(spatial), dtype)

    def num_elements(self) -> int | None:
        n = 1
        for d in self.dims:
            if d is None:
                return None
            n *= d
        return n

    @property
    def rank(self) -> int:
        return len(self.dims)

    def to_json(self) -> dict:
        return {"dims": list(self.dims), "dtype": self.dtype}

    @classmethod
    def from_json(cls, d: dict) -> "TensorShape":
        if d.get("dtype", "f32") not in _ONNX_ELEM:
            raise GraphError(f"unknown tensor dtype {d.get('dtype')!r}")
        return cls(list(d["dims"]), d.get("dtype", "f32"))


@dataclasses.dataclass
class GraphNode:
    node_type: str
    name: str
    output_shape: TensorShape
    attrs: dict | None = None
    extra: dict = dataclasses.field(default_factory=dict)  # axis (concat / softmax), op_type / attributes (custom)

    def __post_init__(self):
        if self.node_type not in NODE_TYPES:
            raise GraphError(f"unknown node type {self.node_type!r}")

    @property
    def onnx_op_type(self) -> str:
        if self.node_type == "activation":
            return _ACT_OP.get(self.attrs["function"], "Activation")
        if self.node_type == "custom":
            return self.extra["op_type"]
        return _ONNX_OP[self.node_type]

    def num_parameters(self) -> int:
        a = self.attrs or {}
        t = self.node_type
        if t == "dense":
            return a["in_features"] * a["out_features"] + (a["out_features"] if a["use_bias"] else 0)
        if t in ("conv2_d", "depthwise_conv2_d"):
            w = a["out_channels"] * (a["in_channels"] // a["groups"]) * a["kernel_h"] * a["kernel_w"]
            return w + (a["out_channels"] if a["use_bias"] else 0)
        if t == "batch_norm":
            return 2 * a["num_features"] if a["affine"] else 0
        if t == "layer_norm":
            n = 1
            for d in a["normalized_shape"]:
                n *= d
            return 2 * n if a["elementwise_affine"] else 0
        if t == "embedding":
            return a["num_embeddings"] * a["embedding_dim"]
        if t == "attention":
            d = a["embed_dim"]
            return 4 * d * d + (4 * d if a["use_bias"] else 0)
        return 0

    def to_json(self) -> dict:
        d = {"node_type": self.node_type, "name": self.name}
        if self.attrs is not None:
            d["attrs"] = self.attrs
        d.update(self.extra)
        d["shape" if self.node_type in ("input", "output") else "output_shape"] = self.output_shape.to_json()
        return d

    @classmethod
    def from_json(cls, d: dict) -> "GraphNode":
        d = dict(d)
        t, name = d.pop("node_type"), d.pop("name")
        shape = TensorShape.from_json(d.pop("shape" if t in ("input", "output") else "output_shape"))
        attrs = d.pop("attrs", None)
        return cls(t, name, shape, attrs, d)


@dataclasses.dataclass
class GraphEdge:
    from_node: str
    to_node: str
    from_slot: int = 0
    to_slot: int = 0

    def to_json(self) -> dict:
        return {"from_node": self.from_node, "from_slot": self.from_slot, "to_node": self.to_node,
                "to_slot": self.to_slot}


@dataclasses.dataclass
class GraphMetadata:
    architecture: str
    framework_version: str = "0.1.0"
    graph_format_version: str = GRAPH_FORMAT_VERSION
    description: str | None = None
    extra: dict = dataclasses.field(default_factory=dict)


class ModelGraph:
    def __init__(self, metadata: GraphMetadata):
        self.metadata = metadata
        self._nodes: list[GraphNode] = []
        self._edges: list[GraphEdge] = []

    # mutation
    def add_node(self, node: GraphNode) -> None:
        if self.find_node(node.name) is not None:
            raise GraphError(f"duplicate node name {node.name!r}")
        self._nodes.append(node)

    def add_edge(self, edge: GraphEdge) -> None:
        for n in (edge.from_node, edge.to_node):
            if self.find_node(n) is None:
                raise GraphError(f"edge references unknown node {n!r}")
        self._edges.append(edge)

    # queries
    @property
    def nodes(self) -> list[GraphNode]:
        return list(self._nodes)

    @property
    def edges(self) -> list[GraphEdge]:
        return list(self._edges)

    def find_node(self, name: str) -> GraphNode | None:
        return next((n for n in self._nodes if n.name == name), None)

    def outgoing_edges(self, name: str) -> list[GraphEdge]:
        return [e for e in self._edges if e.from_node == name]

    def incoming_edges(self, name: str) -> list[GraphEdge]:
        return sorted((e for e in self._edges if e.to_node == name), key=lambda e: e.to_slot)

    def total_parameters(self) -> int:
        return sum(n.num_parameters() for n in self._nodes)

    def topological_order(self) -> list[str]:
        indeg = {n.name: 0 for n in self._nodes}
        for e in self._edges:
            indeg[e.to_node] += 1
        ready = [n.name for n in self._nodes if indeg[n.name] == 0]
        out = []
        while ready:
            u = ready.pop(0)
            out.append(u)
            for e in self.outgoing_edges(u):
                indeg[e.to_node] -= 1
                if indeg[e.to_node] == 0:
                    ready.append(e.to_node)
        if len(out) != len(self._nodes):
            raise GraphError("the graph has a cycle")
        return out

    def validate(self) -> None:
        names = [n.name for n in self._nodes]
        if len(set(names)) != len(names):
            raise GraphError("duplicate node names")
        known = set(names)
        for e in self._edges:
            if e.from_node not in known or e.to_node not in known:
                raise GraphError(f"edge {e.from_node!r} -> {e.to_node!r} references an unknown node")
        if not any(n.node_type == "input" for n in self._nodes):
            raise GraphError("the graph needs at least one input node")
        if not any(n.node_type == "output" for n in self._nodes):
            raise GraphError("the graph needs at least one output node")
        self.topological_order()

    # JSON
    def to_json(self) -> dict:
        return {"metadata": dataclasses.asdict(self.metadata), "nodes": [n.to_json() for n in self._nodes],
                "edges": [e.to_json() for e in self._edges]}

    def export_to_json(self) -> str:
        return json.dumps(self.to_json(), indent=2)

    @classmethod
    def import_from_json(cls, text: str) -> "ModelGraph":
        d = json.loads(text)
        g = cls(GraphMetadata(**d["metadata"]))
        for n in d["nodes"]:
            g.add_node(GraphNode.from_json(n))
        for e in d["edges"]:
            g.add_edge(GraphEdge(e["from_node"], e["to_node"], e.get("from_slot", 0), e.get("to_slot", 0)))
        return g

    def save_to_file(self, path) -> None:
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(self.export_to_json())

    @classmethod
    def load_from_file(cls, path) -> "ModelGraph":
        return cls.import_from_json(Path(path).read_text())

    def export_onnx_like(self) -> dict:
        """An ONNX ModelProto laid out as JSON (ir_version 8, opset 17): graph inputs / outputs with
        tensor types, one node per operator with its inputs named after the producing nodes, and a
        value_info entry per intermediate tensor."""

        def type_proto(s: TensorShape):
            dims = [{"dim_value": v} if v is not None else {"dim_param": "batch_size"} for v in s.dims]
            return {"tensor_type": {"elem_type": _ONNX_ELEM[s.dtype], "shape": {"dim": dims}}}

        inputs, outputs, nodes, vinfo = [], [], [], []
        for n in self._nodes:
            tp = type_proto(n.output_shape)
            if n.node_type == "input":
                inputs.append({"name": n.name, "type": tp})
            elif n.node_type == "output":
                outputs.append({"name": n.name, "type": tp})
            else:
                attrs = [{"name": k, "value": v} for k, v in sorted((n.attrs or {}).items())]
                attrs += [{"name": k, "value": v} for k, v in sorted(n.extra.items()) if k != "op_type"]
                nodes.append({"op_type": n.onnx_op_type, "name": n.name,
                              "input": [e.from_node for e in self.incoming_edges(n.name)], "output": [n.name],
                              "attribute": attrs})
                vinfo.append({"name": n.name, "type": tp})
        doc = self.metadata.description or f"{self.metadata.architecture} model graph"
        return {"ir_version": 8, "opset_import": [{"domain": "", "version": 17}], "model_version": 1,
                "producer_name": "scirs_b200", "producer_version": self.metadata.framework_version,
                "domain": "ai.onnx", "doc_string": doc,
                "graph": {"name": self.metadata.architecture, "doc_string": doc, "input": inputs, "output": outputs,
                          "node": nodes, "value_info": vinfo}}


class ModelGraphBuilder:
    """Fluent construction; `chain(a, b)` adds the edge a:0 -> b:0, `build()` validates."""

    def __init__(self, architecture: str):
        self._g = ModelGraph(GraphMetadata(architecture))
        self._pending: list[GraphEdge] = []

    def _add(self, node):
        self._g.add_node(node)
        return self

    def input(self, name, shape: TensorShape):
        return self._add(GraphNode("input", name, shape))

    def output(self, name, shape: TensorShape):
        return self._add(GraphNode("output", name, shape))

    def dense(self, name, in_features, out_features, use_bias=True, batch=None):
        return self._add(GraphNode("dense", name, TensorShape([batch, out_features]),
                                   {"in_features": in_features, "out_features": out_features, "use_bias": use_bias}))

    def activation(self, name, function, shape: TensorShape, alpha=None):
        return self._add(GraphNode("activation", name, shape, {"function": function, "alpha": alpha}))

    def conv2d(self, name, in_channels, out_channels, kernel, stride=1, padding=0, groups=1, use_bias=True,
               output_shape: TensorShape | None = None):
        attrs = {"in_channels": in_channels, "out_channels": out_channels, "kernel_h": kernel, "kernel_w": kernel,
                 "stride_h": stride, "stride_w": stride,
                 "padding": {"top": padding, "bottom": padding, "left": padding, "right": padding},
                 "dilation": 1, "groups": groups, "use_bias": use_bias}
        kind = "depthwise_conv2_d" if groups > 1 and groups == in_channels else "conv2_d"
        return self._add(GraphNode(kind, name, output_shape or TensorShape([None, out_channels, None, None]), attrs))

    def batch_norm(self, name, num_features, eps=1e-5, momentum=0.1, affine=True, shape=None):
        return self._add(GraphNode("batch_norm", name, shape or TensorShape([None, num_features, None, None]),
                                   {"num_features": num_features, "eps": eps, "momentum": momentum,
                                    "affine": affine}))

    def chain(self, a: str, b: str):
        self._pending.append(GraphEdge(a, b))
        return self

    def edge(self, e: GraphEdge):
        self._pending.append(e)
        return self

    def build(self) -> ModelGraph:
        for e in self._pending:
            self._g.add_edge(e)
        self._g.validate()
        return self._g


# ---------------------------------------------------------------------------- capture from PyTorch modules


def _shape_of(meta) -> TensorShape:
    tm = meta.get("tensor_meta") if meta else None
    if tm is None or not hasattr(tm, "shape"):
        return TensorShape([])
    return TensorShape([None] + list(tm.shape[1:]), _TORCH_DT.get(tm.dtype, "f32"))


def _module_node(name: str, m: nn.Module, shape: TensorShape) -> GraphNode:
    pad = lambda p: {"top": p[0], "bottom": p[0], "left": p[1], "right": p[1]}  # noqa: E731
    two = lambda v: v if isinstance(v, tuple) else (v, v)  # noqa: E731
    from ..models import architectures as A

    if isinstance(m, A.KernelLinear):  # the framework-kernel layers keep their torch attributes
        return GraphNode("dense", name, shape, {"in_features": m.in_features, "out_features": m.out_features,
                                                "use_bias": m.bias is not None})
    if isinstance(m, A.KernelConv2d):
        kh, kw = two(m.kernel_size)
        return GraphNode("conv2_d", name, shape, {
            "in_channels": m.in_channels, "out_channels": m.out_channels, "kernel_h": kh, "kernel_w": kw,
            "stride_h": two(m.stride)[0], "stride_w": two(m.stride)[1], "padding": pad(two(m.padding)),
            "dilation": two(m.dilation)[0], "groups": 1, "use_bias": m.bias is not None})
    if isinstance(m, A.KernelLayerNorm):
        return GraphNode("layer_norm", name, shape, {"normalized_shape": list(m.normalized_shape), "eps": m.eps,
                                                     "elementwise_affine": True})
    if isinstance(m, A.KernelPool2d):
        k, p = two(m.kernel_size), two(m.padding)
        st = two(m.stride if m.stride is not None else m.kernel_size)
        return GraphNode("max_pool2_d" if m.is_max else "avg_pool2_d", name, shape,
                         {"kernel_h": k[0], "kernel_w": k[1], "stride_h": st[0], "stride_w": st[1],
                          "padding": pad(p)})
    if isinstance(m, nn.Linear):
        return GraphNode("dense", name, shape, {"in_features": m.in_features, "out_features": m.out_features,
                                                "use_bias": m.bias is not None})
    if isinstance(m, nn.Conv2d):
        kh, kw = m.kernel_size
        p = m.padding if isinstance(m.padding, tuple) else (0, 0)
        attrs = {"in_channels": m.in_channels, "out_channels": m.out_channels, "kernel_h": kh, "kernel_w": kw,
                 "stride_h": m.stride[0], "stride_w": m.stride[1], "padding": pad(p), "dilation": m.dilation[0],
                 "groups": m.groups, "use_bias": m.bias is not None}
        kind = "depthwise_conv2_d" if m.groups > 1 and m.groups == m.in_channels else "conv2_d"
        return GraphNode(kind, name, shape, attrs)
    if isinstance(m, nn.modules.batchnorm._BatchNorm):
        return GraphNode("batch_norm", name, shape, {"num_features": m.num_features, "eps": m.eps,
                                                     "momentum": m.momentum or 0.0, "affine": m.affine})
    if isinstance(m, nn.LayerNorm):
        return GraphNode("layer_norm", name, shape, {"normalized_shape": list(m.normalized_shape), "eps": m.eps,
                                                     "elementwise_affine": m.elementwise_affine})
    acts = {nn.ReLU: "relu", nn.Sigmoid: "sigmoid", nn.Tanh: "tanh", nn.GELU: "gelu", nn.LeakyReLU: "leaky_relu",
            nn.ELU: "elu", nn.SiLU: "silu", nn.ReLU6: "relu6", nn.Hardswish: "hardswish", nn.Mish: "mish"}
    for cls, fn in acts.items():
        if isinstance(m, cls):
            alpha = getattr(m, "negative_slope", None) or getattr(m, "alpha", None)
            return GraphNode("activation", name, shape, {"function": fn, "alpha": alpha})
    if isinstance(m, (nn.MaxPool2d, nn.AvgPool2d)):
        k, s, p = two(m.kernel_size), two(m.stride if m.stride is not None else m.kernel_size), two(m.padding)
        kind = "max_pool2_d" if isinstance(m, nn.MaxPool2d) else "avg_pool2_d"
        return GraphNode(kind, name, shape, {"kernel_h": k[0], "kernel_w": k[1], "stride_h": s[0], "stride_w": s[1],
                                             "padding": pad(p)})
    if isinstance(m, nn.AdaptiveAvgPool2d) and two(m.output_size) == (1, 1):
        return GraphNode("global_avg_pool", name, shape)
    if isinstance(m, nn.Dropout):
        return GraphNode("dropout", name, shape, {"p": m.p})
    if isinstance(m, nn.Flatten):
        return GraphNode("flatten", name, shape)
    if isinstance(m, nn.Embedding):
        return GraphNode("embedding", name, shape, {"num_embeddings": m.num_embeddings,
                                                    "embedding_dim": m.embedding_dim, "padding_idx": m.padding_idx})
    if isinstance(m, nn.MultiheadAttention):
        return GraphNode("attention", name, shape, {"embed_dim": m.embed_dim, "num_heads": m.num_heads,
                                                    "attn_dropout": m.dropout, "use_bias": m.in_proj_bias is not None})
    if isinstance(m, nn.Softmax):
        return GraphNode("softmax", name, shape, extra={"axis": m.dim if m.dim is not None else -1})
    return GraphNode("custom", name, shape, extra={"op_type": type(m).__name__, "attributes": {}})


_FUNCS = {operator.add: "add", torch.add: "add", torch.cat: "concat", torch.flatten: "flatten",
          torch.relu: ("activation", "relu"), torch.sigmoid: ("activation", "sigmoid"),
          torch.tanh: ("activation", "tanh"), torch.nn.functional.relu: ("activation", "relu"),
          torch.nn.functional.gelu: ("activation", "gelu"), torch.nn.functional.silu: ("activation", "silu"),
          torch.softmax: "softmax", torch.nn.functional.softmax: "softmax"}


def from_module(module: nn.Module, example_input: torch.Tensor, architecture: str | None = None) -> ModelGraph:
    """Captures a module's graph with torch.fx (leaf modules become typed nodes, supported functions
    become add / concat / flatten / activation / softmax nodes, anything else a custom node) and fills
    every output shape by running the example input through it (batch dimension recorded as unknown)."""
    from torch.fx import GraphModule, Tracer
    from torch.fx.passes.shape_prop import ShapeProp

    from ..models import architectures as A

    kernel_layers = (A.KernelLinear, A.KernelConv2d, A.KernelLayerNorm, A.KernelPool2d)

    class _Tracer(Tracer):
        def is_leaf_module(self, m, qualname):
            return isinstance(m, kernel_layers) or super().is_leaf_module(m, qualname)

    gm = GraphModule(module, _Tracer().trace(module))
    ShapeProp(gm).propagate(example_input)
    g = ModelGraph(GraphMetadata(architecture or type(module).__name__))
    mods = dict(gm.named_modules())
    for n in gm.graph.nodes:
        shape = _shape_of(n.meta)
        if n.op == "placeholder":
            g.add_node(GraphNode("input", n.name, shape))
        elif n.op == "output":
            srcs = _flat_args((n.args[0],))
            g.add_node(GraphNode("output", "output", _shape_of(srcs[0].meta if srcs else None)))
            for slot, src in enumerate(srcs):
                g.add_edge(GraphEdge(src.name, "output", 0, slot))
            continue
        elif n.op == "call_module":
            g.add_node(_module_node(n.name, mods[n.target], shape))
        elif n.op in ("call_function", "call_method"):
            kind = _FUNCS.get(n.target) if n.op == "call_function" else None
            if kind is None and n.op == "call_method" and n.target in ("view", "reshape", "flatten"):
                kind = "flatten" if n.target == "flatten" else "reshape"
            if isinstance(kind, tuple):
                g.add_node(GraphNode("activation", n.name, shape, {"function": kind[1], "alpha": None}))
            elif kind == "add":
                g.add_node(GraphNode("add", n.name, shape, {"learnable_scale": False}))
            elif kind == "concat":
                g.add_node(GraphNode("concat", n.name, shape, extra={"axis": n.kwargs.get("dim", n.args[1] if len(
                    n.args) > 1 else 0)}))
            elif kind == "softmax":
                g.add_node(GraphNode("softmax", n.name, shape, extra={"axis": n.kwargs.get("dim", -1)}))
            elif kind == "reshape":
                g.add_node(GraphNode("reshape", n.name, shape, {"shape": [d if d is not None else -1
                                                                          for d in shape.dims]}))
            elif kind == "flatten":
                g.add_node(GraphNode("flatten", n.name, shape))
            else:
                tname = getattr(n.target, "__name__", str(n.target))
                g.add_node(GraphNode("custom", n.name, shape, extra={"op_type": tname, "attributes": {}}))
        else:  # get_attr: a constant / parameter read
            g.add_node(GraphNode("custom", n.name, shape, extra={"op_type": "Constant", "attributes": {}}))
        slot = 0
        for a in _flat_args(n.args) + _flat_args(tuple(n.kwargs.values())):
            g.add_edge(GraphEdge(a.name, n.name, 0, slot))
            slot += 1
    g.validate()
    return g


def _flat_args(args) -> list:
    out = []
    for a in args:
        if isinstance(a, torch.fx.Node):
            out.append(a)
        elif isinstance(a, (list, tuple)):
            out.extend(_flat_args(a))
    return out
