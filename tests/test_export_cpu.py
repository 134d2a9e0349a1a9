"""ONNX export: protobuf and JSON round trips, and the exported graph
reproduces the model (reference interpreter)."""
import torch

from scirs_b200.export import OnnxModel, export_sequential
from scirs_b200.nn import conv as C
from scirs_b200.nn import layers as L
from scirs_b200.nn.sequential import Sequential


def _mlp():
    m = Sequential()
    m.add(L.Dense(12, 16, "relu", seed=1))
    m.add(L.LayerNorm(16))
    m.add(L.Dense(16, 8, seed=2))
    m.add(L.GELU())
    m.add(L.Dropout(0.3))
    m.add(L.Dense(8, 4, "softmax", seed=3))
    return m


def _cnn():
    m = Sequential()
    m.add(C.Conv2D(3, 4, 3, 1, 1))
    m.add(L.BatchNorm(4))
    m.add(L.ReLU())
    m.add(C.MaxPool2D(2))
    m.add(C.Conv2D(4, 6, 3))
    m.add(C.GlobalAvgPool2D())
    m.add(L.Dense(6, 3, seed=4))
    return m


def test_mlp_export_matches_model():
    m = _mlp()
    m.eval()
    onnx = export_sequential(m, [12])
    x = torch.randn(5, 12)
    ref = m(x)
    assert torch.allclose(onnx.run(x), ref, atol=1e-5)
    back = OnnxModel.from_bytes(onnx.to_bytes())
    assert [n.op_type for n in back.graph.nodes] == [n.op_type for n in onnx.graph.nodes]
    assert back.graph.nodes[0].attrs["transB"] == 1 and back.opset == onnx.opset
    assert torch.allclose(back.run(x), ref, atol=1e-5)
    j = OnnxModel.from_json(onnx.to_json())
    assert "Gemm" in onnx.to_json() and torch.allclose(j.run(x), ref, atol=1e-5)


def test_cnn_export_matches_model(tmp_path):
    m = _cnn()
    m.train()
    m(torch.randn(8, 3, 10, 10))  # populate BatchNorm running statistics
    m.eval()
    onnx = export_sequential(m, [3, 10, 10])
    x = torch.randn(2, 3, 10, 10)
    ref = m(x)
    p = tmp_path / "cnn.onnx"
    onnx.save(str(p))
    back = OnnxModel.from_bytes(p.read_bytes())
    assert back.graph.inputs[0].shape == ["N", 3, 10, 10]
    assert torch.allclose(back.run(x), ref, atol=1e-4)
