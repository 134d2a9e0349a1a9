"""Model-graph IR: builder validation, JSON round trips in the reference's
layout, the ONNX-style envelope, parameter counts and graphs captured from
PyTorch modules (a residual block keeps both branches)."""
import json

import pytest
import torch
import torch.nn as nn

from scirs_b200.export import model_graph as MG
from scirs_b200.models import architectures as A


def _mlp_graph():
    return (MG.ModelGraphBuilder("MLP").input("x", MG.TensorShape.with_batch_dim([784]))
            .dense("fc1", 784, 128).activation("act", "relu", MG.TensorShape([None, 128]))
            .dense("fc2", 128, 10).output("y", MG.TensorShape([None, 10]))
            .chain("x", "fc1").chain("fc1", "act").chain("act", "fc2").chain("fc2", "y").build())


def test_builder_json_round_trip_and_counts(tmp_path):
    g = _mlp_graph()
    assert g.total_parameters() == 784 * 128 + 128 + 128 * 10 + 10
    assert g.topological_order() == ["x", "fc1", "act", "fc2", "y"]
    d = json.loads(g.export_to_json())
    assert d["nodes"][0] == {"node_type": "input", "name": "x", "shape": {"dims": [None, 784], "dtype": "f32"}}
    assert d["nodes"][1]["attrs"] == {"in_features": 784, "out_features": 128, "use_bias": True}
    assert d["edges"][0] == {"from_node": "x", "from_slot": 0, "to_node": "fc1", "to_slot": 0}
    g.save_to_file(tmp_path / "sub" / "g.json")
    back = MG.ModelGraph.load_from_file(tmp_path / "sub" / "g.json")
    assert back.to_json() == g.to_json()
    assert [e.to_node for e in back.outgoing_edges("fc1")] == ["act"]


def test_validation_errors():
    b = MG.ModelGraphBuilder("bad").input("x", MG.TensorShape([None, 4]))
    with pytest.raises(MG.GraphError, match="output"):
        b.build()
    g = MG.ModelGraph(MG.GraphMetadata("g"))
    g.add_node(MG.GraphNode("input", "x", MG.TensorShape([1])))
    with pytest.raises(MG.GraphError, match="duplicate"):
        g.add_node(MG.GraphNode("input", "x", MG.TensorShape([1])))
    with pytest.raises(MG.GraphError, match="unknown node"):
        g.add_edge(MG.GraphEdge("x", "nope"))
    with pytest.raises(MG.GraphError, match="unknown node type"):
        MG.GraphNode("warp_drive", "w", MG.TensorShape([1]))
    with pytest.raises(MG.GraphError, match="dtype"):
        MG.TensorShape.from_json({"dims": [1], "dtype": "q7"})
    g.add_node(MG.GraphNode("activation", "a", MG.TensorShape([1]), {"function": "relu", "alpha": None}))
    g.add_node(MG.GraphNode("output", "y", MG.TensorShape([1])))
    g.add_edge(MG.GraphEdge("a", "a"))
    with pytest.raises(MG.GraphError, match="cycle"):
        g.validate()


def test_onnx_like_envelope():
    o = _mlp_graph().export_onnx_like()
    assert o["ir_version"] == 8 and o["opset_import"] == [{"domain": "", "version": 17}]
    gr = o["graph"]
    assert [n["op_type"] for n in gr["node"]] == ["Gemm", "Relu", "Gemm"]
    assert gr["node"][2]["input"] == ["act"] and gr["input"][0]["name"] == "x"
    assert gr["input"][0]["type"]["tensor_type"]["shape"]["dim"][0] == {"dim_param": "batch_size"}
    assert gr["output"][0]["type"]["tensor_type"]["elem_type"] == 1


class _Res(nn.Module):
    def __init__(self):
        super().__init__()
        self.conv = nn.Conv2d(8, 8, 3, padding=1, bias=False)
        self.bn = nn.BatchNorm2d(8)
        self.pool = nn.AdaptiveAvgPool2d(1)
        self.fc = nn.Linear(8, 4)

    def forward(self, x):
        y = torch.relu(self.bn(self.conv(x))) + x
        return torch.softmax(self.fc(torch.flatten(self.pool(y), 1)), dim=-1)


def test_capture_from_module_keeps_residual_and_shapes():
    m = _Res().eval()
    g = MG.from_module(m, torch.randn(2, 8, 6, 6), "ResBlock")
    types = {n.name: n.node_type for n in g.nodes}
    assert types["conv"] == "conv2_d" and types["bn"] == "batch_norm" and types["relu"] == "activation"
    assert types["add"] == "add" and types["pool"] == "global_avg_pool" and types["flatten"] == "flatten"
    assert types["softmax"] == "softmax" and types["fc"] == "dense"
    assert sorted(e.from_node for e in g.incoming_edges("add")) == ["relu", "x"]  # both branches
    assert g.find_node("conv").output_shape.dims == [None, 8, 6, 6]
    assert g.find_node("fc").output_shape.dims == [None, 4]
    assert g.total_parameters() == sum(p.numel() for p in m.parameters())
    back = MG.ModelGraph.import_from_json(g.export_to_json())
    assert back.topological_order() == g.topological_order()


def test_capture_zoo_model():
    cfg = A.ResNetConfig.resnet18(3, 10)
    m = cfg.build().eval()
    g = MG.from_module(m, torch.randn(1, 3, 32, 32), "ResNet")
    assert g.total_parameters() == sum(p.numel() for p in m.parameters())
    assert sum(n.node_type == "add" for n in g.nodes) == 8  # one residual add per basic block
    assert g.find_node("output").output_shape.dims == [None, 10]
