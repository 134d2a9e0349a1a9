"""Static-graph tracing: builder, optimizer (dead nodes, Linear -> ReLU
fusion), executor with the reference's weight-map keys, and tracing of an
nn.Sequential, checked against the module itself (float64, CPU)."""
import pytest
import torch

from scirs_b200.nn import tracing as T


def test_builder_executor_and_weight_keys():
    gb = T.GraphBuilder()
    x = gb.input(T.TensorSpec([2, 3]))
    h = gb.linear(x, 3, 4)
    r = gb.relu(h)
    dead = gb.sigmoid(r)  # not an output: removed by optimize
    s = gb.softmax(r, 1)
    g = gb.build([s])
    assert g.input_node_ids == [0] and g.output_node_ids == [s.id] and g.num_nodes() == 5
    assert g.get_node(h.id).outputs == [r.id] and g.get_node(99) is None
    torch.manual_seed(0)
    W, b = torch.randn(4, 3, dtype=torch.float64), torch.randn(4, dtype=torch.float64)
    wm = {f"linear_{h.id}_weight": W.reshape(-1).tolist(), f"linear_{h.id}_bias": b.tolist()}
    xin = torch.randn(2, 3, dtype=torch.float64)
    ref = torch.softmax(torch.relu(xin @ W.t() + b), dim=1)
    out = T.GraphExecutor(g, wm).run([xin])[0]
    assert torch.allclose(out, ref)
    og = T.optimize(g)
    kinds = [n.op_type for n in og.nodes]
    assert T.OpType.FUSED_LINEAR_RELU in kinds and T.OpType.RELU not in kinds and T.OpType.SIGMOID not in kinds
    assert og.get_node(h.id).op_type is T.OpType.FUSED_LINEAR_RELU
    assert torch.allclose(T.GraphExecutor(og, wm).run([xin.reshape(-1).tolist()])[0], ref)
    og2 = T.StaticGraph.from_json(og.to_json())
    assert [n.op_type for n in og2.nodes] == kinds
    assert torch.allclose(T.GraphExecutor(og2, wm).run([xin])[0], ref)
    with pytest.raises(ValueError):
        T.GraphExecutor(g, {}).run([xin])
    with pytest.raises(ValueError):
        T.GraphExecutor(g, wm).run([])


def test_binary_reshape_layernorm_and_output_linear_not_fused():
    gb = T.GraphBuilder()
    a = gb.input(T.TensorSpec([2, 4]))
    c = gb.input(T.TensorSpec([2, 4]))
    m = gb.mul(gb.add(a, c), c)
    ln = gb.layer_norm(m, 1e-6)
    rs = gb.reshape(ln, [4, 2])
    lin = gb.linear(rs, 2, 2)
    g = gb.build([lin, gb.tanh(lin)])
    torch.manual_seed(1)
    A, C = torch.randn(2, 4, dtype=torch.float64), torch.randn(2, 4, dtype=torch.float64)
    gam, bet = torch.rand(4, dtype=torch.float64) + 0.5, torch.randn(4, dtype=torch.float64)
    W, b = torch.randn(2, 2, dtype=torch.float64), torch.randn(2, dtype=torch.float64)
    wm = {f"layer_norm_{ln.id}_gamma": gam.tolist(), f"layer_norm_{ln.id}_beta": bet.tolist(),
          f"linear_{lin.id}_weight": W.reshape(-1).tolist(), f"linear_{lin.id}_bias": b.tolist()}
    y = torch.nn.functional.layer_norm((A + C) * C, (4,), gam, bet, 1e-6).reshape(4, 2) @ W.t() + b
    o1, o2 = T.GraphExecutor(T.optimize(g), wm).run([A, C])
    assert torch.allclose(o1, y) and torch.allclose(o2, torch.tanh(y))


def test_trace_sequential_matches_module():
    torch.manual_seed(2)
    model = torch.nn.Sequential(torch.nn.Flatten(), torch.nn.Linear(12, 16), torch.nn.ReLU(),
                                torch.nn.LayerNorm(16), torch.nn.Linear(16, 8), torch.nn.Tanh(),
                                torch.nn.Linear(8, 5), torch.nn.Softmax(dim=-1)).double()
    x = torch.randn(3, 3, 4, dtype=torch.float64)
    g, wm = T.trace_sequential(model, [3, 3, 4])
    assert any(n.op_type is T.OpType.FUSED_LINEAR_RELU for n in g.nodes)
    with torch.no_grad():
        assert torch.allclose(T.GraphExecutor(g, wm).run([x])[0], model(x))
    g0, _ = T.trace_sequential(model, [3, 3, 4], T.TraceConfig(optimize=False))
    assert not any(n.op_type is T.OpType.FUSED_LINEAR_RELU for n in g0.nodes)
