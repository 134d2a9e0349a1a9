"""ONNX export of autograd graphs (the exported model computes what the
graph computes, also after a protobuf / JSON round trip) and the graph
builder's validation."""
import numpy as np
import pytest
import torch

from scirs_b200.autograd import VariableEnvironment
from scirs_b200.autograd import ops as T
from scirs_b200.export.onnx import OnnxModel, OnnxTensor
from scirs_b200.export.onnx_graph import (OnnxGraphBuilder, export_graph, onnx_to_tensor, run_onnx,
                                          tensor_to_onnx)


def _mlp_env():
    g = torch.Generator().manual_seed(0)
    env = VariableEnvironment()
    env.name("w1").set(torch.randn(8, 16, generator=g))
    env.name("b1").set(torch.randn(16, generator=g))
    env.name("w2").set(torch.randn(16, 4, generator=g))
    return env


def test_export_mlp_graph_matches_evaluation():
    env = _mlp_env()
    x0 = torch.randn(5, 8, generator=torch.Generator().manual_seed(1))

    def body(ctx):
        x = ctx.placeholder("x", [-1, 8])
        h = T.gelu(T.matmul(x, ctx.variable("w1")) + ctx.variable("b1"))
        h = T.layer_norm(h, ctx.constant(torch.ones(16)), ctx.constant(torch.zeros(16)))
        z = T.matmul(T.swish(h), ctx.variable("w2"))
        p = T.softmax(z, axis=-1)
        s = T.reduce_mean(T.square(z) * 0.5 - T.log(p + 1e-6), axes=[1], keep_dims=False)
        m = export_graph([p, s], {"x": x0})
        want = ctx.evaluator().torch().push(p).push(s).feed("x", x0).run()
        return m, want

    m, want = env.run(body)
    got = run_onnx(m, {"x": x0})
    for a, b in zip(got, want):
        assert torch.allclose(a, b, atol=1e-5), (a, b)
    # protobuf round trip
    m2 = OnnxModel.from_bytes(m.to_bytes())
    assert [n.op_type for n in m2.graph.nodes] == [n.op_type for n in m.graph.nodes]
    for a, b in zip(run_onnx(m2, {"x": x0}), want):
        assert torch.allclose(a, b, atol=1e-5)
    # JSON round trip
    m3 = OnnxModel.from_json(m.to_json())
    for a, b in zip(run_onnx(m3, {"x": x0}), want):
        assert torch.allclose(a, b, atol=1e-5)


def test_export_shape_ops_and_conv():
    g = torch.Generator().manual_seed(2)
    x0 = torch.randn(2, 3, 8, 8, generator=g)
    w0 = torch.randn(4, 3, 3, 3, generator=g)

    def body(ctx):
        x = ctx.placeholder("x", [2, 3, 8, 8])
        y = T.relu(T.conv2d(x, ctx.constant(w0), stride=1, padding=1))
        y = T.max_pool2d(y, 2, 2)
        y = T.reshape(y, [2, -1])
        y = T.transpose(y)
        y = T.concat([y, y * 2.0], axis=1)
        y = T.clip(T.expand_dims(y, 0), -1.0, 1.0)
        m = export_graph(y, {"x": x0})
        return m, ctx.evaluator().torch().push(y).feed("x", x0).run()[0]

    from scirs_b200.autograd import run

    m, want = run(body)
    got = run_onnx(m, {"x": x0})[0]
    assert got.shape == want.shape and torch.allclose(got, want, atol=1e-5)


def test_export_rejects_gradient_nodes():
    from scirs_b200.autograd import grad, run

    def body(ctx):
        x = ctx.placeholder("x", [3])
        y = T.reduce_sum(T.square(x))
        (gx,) = grad([y], [x])
        with pytest.raises(NotImplementedError):
            export_graph(gx, {"x": torch.ones(3)})

    run(body)


def test_builder_validates_and_runs():
    b = (OnnxGraphBuilder("tiny").add_input("x", [2, 3]).add_output("y", [2, 4])
         .add_initializer(tensor_to_onnx("w", torch.ones(3, 4)))
         .add_initializer(tensor_to_onnx("c", torch.full((4,), 0.5)))
         .add_gemm("g", "x", "w", "c", "h")
         .add_relu("r", "h", "y"))
    m = b.model()
    out = run_onnx(m, {"x": torch.tensor([[1.0, -2.0, 0.5], [-1.0, -1.0, -1.0]])})[0]
    assert torch.allclose(out, torch.tensor([[0.0, 0.0, 0.0, 0.0], [0.0, 0.0, 0.0, 0.0]]))
    bad = OnnxGraphBuilder("bad").add_input("x", [1]).add_output("y", [1]).add_relu("r", "nope", "y")
    with pytest.raises(ValueError, match="undefined"):
        bad.build()


def test_tensor_conversions():
    t = torch.arange(6.0).reshape(2, 3)
    ot = tensor_to_onnx("t", t)
    assert isinstance(ot, OnnxTensor) and ot.dims == [2, 3]
    assert torch.equal(onnx_to_tensor(ot), t)
    it = tensor_to_onnx("i", torch.tensor([1, 2, 3]))
    assert it.data_type == 7 and onnx_to_tensor(it).tolist() == [1, 2, 3]
    assert np.allclose(onnx_to_tensor(ot).numpy(), t.numpy())
