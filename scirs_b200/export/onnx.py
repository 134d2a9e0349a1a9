"""ONNX export of layer models (real ONNX protobuf, plus a JSON form).

The protobuf encoder writes the ONNX wire format directly (ModelProto ->
GraphProto -> NodeProto / TensorProto / ValueInfoProto, field numbers of the
public onnx.proto), so exported files open in any ONNX runtime without the
`onnx` package being installed here. `OnnxModel.to_json` / `from_json` keep
the reference's JSON interchange form, and `run` is a small reference
interpreter (PyTorch ops) used to check an export against the model.

Supported layers (nn.Sequential / scirs_b200.nn.Sequential): Dense (Gemm,
transB=1 over the [out, in] weight), Conv2D (Conv), BatchNorm
(BatchNormalization), LayerNorm (LayerNormalization), activations (Relu,
Sigmoid, Tanh, Softmax, Gelu, LeakyRelu, Elu), Flatten, MaxPool2D /
AvgPool2D / GlobalAvgPool2D, Dropout (exported as Identity).

Reference parity: scirs2-neural/src/export/onnx.rs:64-560 (OnnxNode,
OnnxTensor, OnnxValueInfo, OnnxGraph, OnnxModel, export_linear /
export_conv2d / export_activation / export_batchnorm / export_sequential).
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field

import torch

FLOAT, INT64 = 1, 7  # TensorProto data types
OPSET = 20


# ---------------------------------------------------------------- graph IR
@dataclass
class OnnxNode:
    op_type: str
    name: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)

    def with_attr(self, k, v):
        self.attrs[k] = v
        return self


@dataclass
class OnnxTensor:
    name: str
    dims: list
    data: list  # float values (row-major)
    data_type: int = FLOAT

    @staticmethod
    def from_tensor(name: str, t: torch.Tensor) -> "OnnxTensor":
        t = t.detach().float().cpu().contiguous()
        return OnnxTensor(name, list(t.shape), t.reshape(-1).tolist())

    def numel(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    def to_torch(self) -> torch.Tensor:
        dt = torch.int64 if self.data_type == INT64 else torch.float32
        return torch.tensor(self.data, dtype=dt).reshape(self.dims)


@dataclass
class OnnxValueInfo:
    name: str
    elem_type: int
    shape: list  # ints or None (symbolic)


@dataclass
class OnnxGraph:
    name: str = "scirs_b200"
    nodes: list = field(default_factory=list)
    initializers: list = field(default_factory=list)
    inputs: list = field(default_factory=list)
    outputs: list = field(default_factory=list)


@dataclass
class OnnxModel:
    graph: OnnxGraph
    ir_version: int = 9
    opset: int = OPSET
    producer_name: str = "scirs_b200"
    producer_version: str = "0.1.0"

    # ------------------------------------------------------------- JSON
    def to_json(self) -> str:
        g = self.graph
        return json.dumps({
            "ir_version": self.ir_version, "opset_version": self.opset, "producer_name": self.producer_name,
            "producer_version": self.producer_version,
            "graph": {
                "name": g.name,
                "nodes": [vars(n) for n in g.nodes],
                "initializers": [vars(t) for t in g.initializers],
                "inputs": [vars(v) for v in g.inputs],
                "outputs": [vars(v) for v in g.outputs],
            },
        }, indent=2)

    @staticmethod
    def from_json(s: str) -> "OnnxModel":
        d = json.loads(s)
        g = d["graph"]
        graph = OnnxGraph(g["name"], [OnnxNode(**n) for n in g["nodes"]], [OnnxTensor(**t) for t in g["initializers"]],
                          [OnnxValueInfo(**v) for v in g["inputs"]], [OnnxValueInfo(**v) for v in g["outputs"]])
        return OnnxModel(graph, d["ir_version"], d["opset_version"], d["producer_name"], d["producer_version"])

    # ------------------------------------------------------------- protobuf
    def to_bytes(self) -> bytes:
        return _encode_model(self)

    def save(self, path: str):
        with open(path, "wb") as f:
            f.write(self.to_bytes())

    @staticmethod
    def from_bytes(b: bytes) -> "OnnxModel":
        return _decode_model(b)

    # ------------------------------------------------------------- execute
    def run(self, x: torch.Tensor) -> torch.Tensor:
        return run_graph(self.graph, {self.graph.inputs[0].name: x})[self.graph.outputs[0].name]


# ---------------------------------------------------------------- wire format
def _varint(n: int) -> bytes:
    n &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field_no: int, wire: int) -> bytes:
    return _varint((field_no << 3) | wire)


def _len(field_no: int, payload: bytes) -> bytes:
    return _key(field_no, 2) + _varint(len(payload)) + payload


def _int(field_no: int, v: int) -> bytes:
    return _key(field_no, 0) + _varint(v)


def _str(field_no: int, s: str) -> bytes:
    return _len(field_no, s.encode())


def _enc_attr(name, v) -> bytes:
    # AttributeProto: name=1, f=2, i=3, s=4, floats=7, ints=8, type=20
    b = _str(1, name)
    if isinstance(v, float):
        b += _key(2, 5) + struct.pack("<f", v) + _int(20, 1)
    elif isinstance(v, bool) or isinstance(v, int):
        b += _int(3, int(v)) + _int(20, 2)
    elif isinstance(v, str):
        b += _len(4, v.encode()) + _int(20, 3)
    elif isinstance(v, (list, tuple)) and all(isinstance(e, int) for e in v):
        b += b"".join(_int(8, e) for e in v) + _int(20, 7)
    elif isinstance(v, (list, tuple)):
        b += b"".join(_key(7, 5) + struct.pack("<f", float(e)) for e in v) + _int(20, 6)
    else:
        raise TypeError(f"unsupported attribute {name}={v!r}")
    return b


def _enc_tensor(t: OnnxTensor) -> bytes:
    # TensorProto: dims=1, data_type=2, name=8, raw_data=9 (little-endian)
    b = b"".join(_int(1, d) for d in t.dims) + _int(2, t.data_type) + _str(8, t.name)
    fmt = "<%df" % len(t.data) if t.data_type == FLOAT else "<%dq" % len(t.data)
    return b + _len(9, struct.pack(fmt, *t.data))


def _enc_value_info(v: OnnxValueInfo) -> bytes:
    dims = b""
    for d in v.shape:
        dims += _len(1, _int(1, d) if isinstance(d, int) else _str(2, d or "N"))
    tensor_type = _int(1, v.elem_type) + _len(2, dims)
    return _str(1, v.name) + _len(2, _len(1, tensor_type))


def _enc_node(n: OnnxNode) -> bytes:
    b = b"".join(_str(1, i) for i in n.inputs) + b"".join(_str(2, o) for o in n.outputs)
    b += _str(3, n.name) + _str(4, n.op_type)
    b += b"".join(_len(5, _enc_attr(k, v)) for k, v in n.attrs.items())
    return b


def _encode_model(m: OnnxModel) -> bytes:
    g = m.graph
    gb = b"".join(_len(1, _enc_node(n)) for n in g.nodes) + _str(2, g.name)
    gb += b"".join(_len(5, _enc_tensor(t)) for t in g.initializers)
    gb += b"".join(_len(11, _enc_value_info(v)) for v in g.inputs)
    gb += b"".join(_len(12, _enc_value_info(v)) for v in g.outputs)
    opset = _str(1, "") + _int(2, m.opset)
    return (_int(1, m.ir_version) + _str(2, m.producer_name) + _str(3, m.producer_version) + _len(7, gb)
            + _len(8, opset))


def _fields(b: bytes):
    i = 0
    while i < len(b):
        k, i = _rd_varint(b, i)
        f, w = k >> 3, k & 7
        if w == 0:
            v, i = _rd_varint(b, i)
        elif w == 2:
            n, i = _rd_varint(b, i)
            v, i = b[i : i + n], i + n
        elif w == 5:
            v, i = b[i : i + 4], i + 4
        elif w == 1:
            v, i = b[i : i + 8], i + 8
        else:
            raise ValueError("unsupported wire type")
        yield f, w, v


def _rd_varint(b, i):
    shift = n = 0
    while True:
        c = b[i]
        i += 1
        n |= (c & 0x7F) << shift
        shift += 7
        if not c & 0x80:
            return n, i


def _decode_model(b: bytes) -> OnnxModel:
    m = OnnxModel(OnnxGraph())
    for f, w, v in _fields(b):
        if f == 1:
            m.ir_version = v
        elif f == 2:
            m.producer_name = v.decode()
        elif f == 3:
            m.producer_version = v.decode()
        elif f == 8:
            m.opset = dict((ff, vv) for ff, _, vv in _fields(v)).get(2, m.opset)
        elif f == 7:
            g = m.graph
            for gf, _, gv in _fields(v):
                if gf == 1:
                    g.nodes.append(_dec_node(gv))
                elif gf == 2:
                    g.name = gv.decode()
                elif gf == 5:
                    g.initializers.append(_dec_tensor(gv))
                elif gf in (11, 12):
                    (g.inputs if gf == 11 else g.outputs).append(_dec_value_info(gv))
    return m


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _dec_node(b):
    n = OnnxNode("", "", [], [])
    for f, _, v in _fields(b):
        if f == 1:
            n.inputs.append(v.decode())
        elif f == 2:
            n.outputs.append(v.decode())
        elif f == 3:
            n.name = v.decode()
        elif f == 4:
            n.op_type = v.decode()
        elif f == 5:
            name, val, ints, floats, typ = None, None, [], [], 0
            for af, aw, av in _fields(v):
                if af == 1:
                    name = av.decode()
                elif af == 2:
                    val = struct.unpack("<f", av)[0]
                elif af == 3:
                    val = _signed(av)
                elif af == 4:
                    val = av.decode()
                elif af == 7:
                    floats.append(struct.unpack("<f", av)[0])
                elif af == 8:
                    ints.append(_signed(av))
                elif af == 20:
                    typ = av
            n.attrs[name] = ints if typ == 7 else (floats if typ == 6 else val)
    return n


def _dec_tensor(b):
    dims, dt, name, raw = [], FLOAT, "", b""
    for f, _, v in _fields(b):
        if f == 1:
            dims.append(v)
        elif f == 2:
            dt = v
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = v
    fmt = "<%df" % (len(raw) // 4) if dt == FLOAT else "<%dq" % (len(raw) // 8)
    return OnnxTensor(name, dims, list(struct.unpack(fmt, raw)), dt)


def _dec_value_info(b):
    name, elem, shape = "", FLOAT, []
    for f, _, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:
            for _, _, tt in _fields(v):
                for tf, _, tv in _fields(tt):
                    if tf == 1:
                        elem = tv
                    elif tf == 2:
                        for _, _, dim in _fields(tv):
                            d = dict((df, dv) for df, _, dv in _fields(dim))
                            shape.append(d[1] if 1 in d else d.get(2, b"N").decode())
    return OnnxValueInfo(name, elem, shape)


# ---------------------------------------------------------------- exporters
def export_linear(w_out_in: torch.Tensor, bias, inp: str, out: str, prefix: str):
    inits = [OnnxTensor.from_tensor(prefix + ".weight", w_out_in)]
    ins = [inp, prefix + ".weight"]
    if bias is not None:
        inits.append(OnnxTensor.from_tensor(prefix + ".bias", bias))
        ins.append(prefix + ".bias")
    node = OnnxNode("Gemm", prefix + "/Gemm", ins, [out], {"transB": 1, "alpha": 1.0, "beta": 1.0})
    return [node], inits


def export_conv2d(w, bias, stride, padding, inp, out, prefix):
    inits = [OnnxTensor.from_tensor(prefix + ".weight", w)]
    ins = [inp, prefix + ".weight"]
    if bias is not None:
        inits.append(OnnxTensor.from_tensor(prefix + ".bias", bias))
        ins.append(prefix + ".bias")
    s = [stride, stride] if isinstance(stride, int) else list(stride)
    p = [padding, padding] if isinstance(padding, int) else list(padding)
    node = OnnxNode("Conv", prefix + "/Conv", ins, [out],
                    {"kernel_shape": list(w.shape[2:]), "strides": s, "pads": [p[0], p[1], p[0], p[1]]})
    return [node], inits


_ACT = {"relu": "Relu", "sigmoid": "Sigmoid", "tanh": "Tanh", "softmax": "Softmax", "gelu": "Gelu"}


def export_activation(kind: str, inp: str, out: str, name: str | None = None):
    op = _ACT[kind.lower()]
    n = OnnxNode(op, name or f"{out}/{op}", [inp], [out])
    if op == "Softmax":
        n.attrs["axis"] = -1
    if op == "Gelu":
        n.attrs["approximate"] = "tanh"
    return n


def export_batchnorm(gamma, beta, mean, var, eps, inp, out, prefix):
    names = [prefix + s for s in (".weight", ".bias", ".running_mean", ".running_var")]
    inits = [OnnxTensor.from_tensor(n, t) for n, t in zip(names, (gamma, beta, mean, var))]
    return [OnnxNode("BatchNormalization", prefix + "/BN", [inp] + names, [out], {"epsilon": float(eps)})], inits


def export_sequential(model, input_shape, name: str = "model") -> OnnxModel:
    """Export a sequential layer model; input_shape without the batch dim."""
    from ..nn import conv as C
    from ..nn import layers as Lr

    layers = list(model.layers()) if hasattr(model, "layers") and callable(model.layers) else list(model)
    g = OnnxGraph(name)
    cur = "input"
    g.inputs.append(OnnxValueInfo("input", FLOAT, ["N"] + list(input_shape)))
    for i, layer in enumerate(layers):
        out = f"t{i}"
        p = f"layers.{i}"
        if isinstance(layer, (Lr.Dense, torch.nn.Linear)):
            w = layer.weight.t() if isinstance(layer, Lr.Dense) else layer.weight  # Dense keeps [in, out]
            nodes, inits = export_linear(w, layer.bias, cur, out, p)
            act = layer.activation() if isinstance(layer, Lr.Dense) else None
            if act:
                mid = out + "_pre"
                nodes[0].outputs = [mid]
                nodes.append(export_activation(act, mid, out))
        elif isinstance(layer, (C.Conv2D, torch.nn.Conv2d)):
            nodes, inits = export_conv2d(layer.weight, layer.bias, layer.stride, layer.padding, cur, out, p)
        elif isinstance(layer, (Lr.BatchNorm, torch.nn.BatchNorm1d, torch.nn.BatchNorm2d)):
            nodes, inits = export_batchnorm(layer.weight, layer.bias, layer.running_mean, layer.running_var,
                                            layer.eps, cur, out, p)
        elif isinstance(layer, (Lr.LayerNorm, torch.nn.LayerNorm)):
            inits = [OnnxTensor.from_tensor(p + ".weight", layer.weight), OnnxTensor.from_tensor(p + ".bias", layer.bias)]
            nodes = [OnnxNode("LayerNormalization", p + "/LN", [cur, p + ".weight", p + ".bias"], [out],
                              {"axis": -1, "epsilon": float(layer.eps)})]
        elif isinstance(layer, (Lr.ReLU, torch.nn.ReLU)):
            nodes, inits = [export_activation("relu", cur, out)], []
        elif isinstance(layer, (Lr.Sigmoid, torch.nn.Sigmoid)):
            nodes, inits = [export_activation("sigmoid", cur, out)], []
        elif isinstance(layer, (Lr.Tanh, torch.nn.Tanh)):
            nodes, inits = [export_activation("tanh", cur, out)], []
        elif isinstance(layer, (Lr.Softmax, torch.nn.Softmax)):
            nodes, inits = [export_activation("softmax", cur, out)], []
        elif isinstance(layer, (Lr.GELU, torch.nn.GELU)):
            nodes, inits = [export_activation("gelu", cur, out)], []
        elif isinstance(layer, Lr.LeakyReLU):
            nodes, inits = [OnnxNode("LeakyRelu", out + "/LeakyRelu", [cur], [out], {"alpha": float(layer.alpha)})], []
        elif isinstance(layer, Lr.ELU):
            nodes, inits = [OnnxNode("Elu", out + "/Elu", [cur], [out], {"alpha": float(layer.alpha)})], []
        elif isinstance(layer, (Lr.Flatten, torch.nn.Flatten)):
            nodes, inits = [OnnxNode("Flatten", out + "/Flatten", [cur], [out], {"axis": 1})], []
        elif isinstance(layer, (Lr.Dropout, torch.nn.Dropout)):
            nodes, inits = [OnnxNode("Identity", out + "/Identity", [cur], [out])], []
        elif isinstance(layer, C.MaxPool2D):
            k, s = layer.kernel_size, layer.stride
            nodes, inits = [OnnxNode("MaxPool", out + "/MaxPool", [cur], [out],
                                     {"kernel_shape": [k, k], "strides": [s, s]})], []
        elif isinstance(layer, C.AvgPool2D):
            k, s = layer.kernel_size, layer.stride
            nodes, inits = [OnnxNode("AveragePool", out + "/AveragePool", [cur], [out],
                                     {"kernel_shape": [k, k], "strides": [s, s]})], []
        elif isinstance(layer, C.GlobalAvgPool2D):
            nodes, inits = [OnnxNode("GlobalAveragePool", out + "/GAP", [cur], [out + "_4d"]),
                            OnnxNode("Flatten", out + "/Flatten", [out + "_4d"], [out], {"axis": 1})], []
        else:
            raise NotImplementedError(f"ONNX export of {type(layer).__name__}")
        g.nodes += nodes
        g.initializers += inits
        cur = out
    g.outputs.append(OnnxValueInfo(cur, FLOAT, ["N", "D"]))
    return OnnxModel(g)


# ---------------------------------------------------------------- interpreter
_ELEMENTWISE = {
    "Add": torch.add, "Sub": torch.sub, "Mul": torch.mul, "Div": torch.div, "Pow": torch.pow, "Neg": torch.neg,
    "Exp": torch.exp, "Log": torch.log, "Sqrt": torch.sqrt, "Abs": torch.abs, "Sin": torch.sin, "Cos": torch.cos,
    "Tan": torch.tan, "Asin": torch.asin, "Acos": torch.acos, "Atan": torch.atan, "Sinh": torch.sinh,
    "Cosh": torch.cosh, "Erf": torch.erf, "Floor": torch.floor, "Ceil": torch.ceil, "Sign": torch.sign,
    "Round": torch.round, "Reciprocal": torch.reciprocal, "Max": torch.maximum, "Min": torch.minimum,
    "Softplus": lambda t: torch.nn.functional.softplus(t), "Selu": lambda t: torch.nn.functional.selu(t),
    "Softsign": lambda t: torch.nn.functional.softsign(t), "HardSwish": lambda t: torch.nn.functional.hardswish(t),
    "Mish": lambda t: torch.nn.functional.mish(t),
}


def _reduce(op, x, axes, keep):
    fn = {"ReduceSum": torch.sum, "ReduceMean": torch.mean, "ReduceProd": None, "ReduceMax": torch.amax,
          "ReduceMin": torch.amin}[op]
    if axes is None:
        if op == "ReduceProd":
            return x.prod()
        return x.max() if op == "ReduceMax" else (x.min() if op == "ReduceMin" else fn(x))
    if op == "ReduceProd":
        for ax in sorted(axes, reverse=True):
            x = x.prod(ax, keepdim=keep)
        return x
    return fn(x, tuple(int(v) for v in axes), keepdim=keep)


def run_graph(graph: OnnxGraph, feeds: dict) -> dict:
    import torch.nn.functional as F

    env = dict(feeds)
    env.update({t.name: t.to_torch() for t in graph.initializers})
    for n in graph.nodes:
        x = [env[i] for i in n.inputs]
        a = n.attrs
        op = n.op_type
        if op == "Gemm":
            w = x[1].t() if a.get("transB") else x[1]
            y = a.get("alpha", 1.0) * (x[0] @ w) + (a.get("beta", 1.0) * x[2] if len(x) > 2 else 0)
        elif op == "Conv":
            p = a.get("pads", [0, 0, 0, 0])
            y = F.conv2d(x[0], x[1], x[2] if len(x) > 2 else None, a.get("strides", [1, 1]), p[:2])
        elif op == "Relu":
            y = torch.relu(x[0])
        elif op == "Sigmoid":
            y = torch.sigmoid(x[0])
        elif op == "Tanh":
            y = torch.tanh(x[0])
        elif op == "Softmax":
            y = torch.softmax(x[0], a.get("axis", -1))
        elif op == "Gelu":
            y = F.gelu(x[0], approximate=a.get("approximate", "none"))
        elif op == "LeakyRelu":
            y = F.leaky_relu(x[0], a.get("alpha", 0.01))
        elif op == "Elu":
            y = F.elu(x[0], a.get("alpha", 1.0))
        elif op == "BatchNormalization":
            y = F.batch_norm(x[0], x[3], x[4], x[1], x[2], False, 0.0, a.get("epsilon", 1e-5))
        elif op == "LayerNormalization":
            y = F.layer_norm(x[0], x[0].shape[-1:], x[1], x[2], a.get("epsilon", 1e-5))
        elif op == "Flatten":
            y = x[0].flatten(a.get("axis", 1))
        elif op == "Identity":
            y = x[0]
        elif op == "MaxPool":
            y = F.max_pool2d(x[0], a["kernel_shape"], a.get("strides"))
        elif op == "AveragePool":
            y = F.avg_pool2d(x[0], a["kernel_shape"], a.get("strides"))
        elif op == "GlobalAveragePool":
            y = x[0].mean(dim=(2, 3), keepdim=True)
        elif op in _ELEMENTWISE:
            y = _ELEMENTWISE[op](*x)
        elif op in ("ReduceSum", "ReduceMean", "ReduceMax", "ReduceMin", "ReduceProd"):
            y = _reduce(op, x[0], x[1].tolist() if len(x) > 1 else None, bool(a.get("keepdims", 1)))
        elif op == "MatMul":
            y = x[0] @ x[1]
        elif op == "Reshape":
            y = x[0].reshape([int(v) for v in x[1].tolist()])
        elif op == "Transpose":
            y = x[0].permute(*a["perm"])
        elif op == "Concat":
            y = torch.cat(x, a["axis"])
        elif op == "Unsqueeze":
            y = x[0]
            for ax in sorted(int(v) for v in x[1].reshape(-1).tolist()):
                y = y.unsqueeze(ax)
        elif op == "Squeeze":
            y = x[0].squeeze(int(x[1].reshape(-1)[0]))
        elif op in ("Softmax", "LogSoftmax"):
            y = (torch.softmax if op == "Softmax" else torch.log_softmax)(x[0], a.get("axis", -1))
        elif op == "Clip":
            y = x[0].clamp(float(x[1]), float(x[2]))
        elif op == "Cast":
            y = x[0].bool() if a.get("to") == 9 else x[0].float()
        elif op == "Where":
            y = torch.where(x[0].bool(), x[1], x[2])
        elif op == "Gather":
            y = torch.index_select(x[0], a.get("axis", 0), x[1].reshape(-1).long())
            if x[1].dim() == 0:
                y = y.squeeze(a.get("axis", 0))
        elif op == "HardSigmoid":
            y = (a.get("alpha", 0.2) * x[0] + a.get("beta", 0.5)).clamp(0, 1)
        else:
            raise NotImplementedError(op)
        env[n.outputs[0]] = y
    return env
