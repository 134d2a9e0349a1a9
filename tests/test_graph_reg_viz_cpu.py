"""Graph layers, activity regularisation and headless visualisation."""
import torch

from scirs_b200.nn import graph as GN
from scirs_b200.nn import regularization as R
from scirs_b200.utils import visualization as V


def _ring(n):
    a = torch.zeros(n, n)
    for i in range(n):
        a[i, (i + 1) % n] = a[(i + 1) % n, i] = 1
    return a


def test_gcn_matches_formula_and_trains():
    torch.manual_seed(0)
    n, fi, fo = 6, 5, 3
    adj, h = _ring(n), torch.randn(n, fi)
    layer = GN.GraphConvLayer(fi, fo, activation="none")
    a = adj + torch.eye(n)
    d = a.sum(1).rsqrt()
    want = (d[:, None] * a * d[None, :]) @ (h @ layer.lin.weight.t()) + layer.bias
    torch.testing.assert_close(layer(h, adj), want)
    layer(h, adj).square().mean().backward()
    assert layer.lin.weight.grad is not None


def test_gat_respects_graph_and_heads():
    torch.manual_seed(0)
    n = 5
    adj = torch.zeros(n, n)
    adj[0, 1] = adj[1, 0] = 1
    gat = GN.GraphAttentionLayer(4, 3, num_heads=2, concat=True, activation="none")
    h = torch.randn(n, 4)
    out = gat(h, adj)
    assert out.shape == (n, 6)
    # node 4 is isolated: attends only to itself
    z = gat.W(h).view(n, 2, 3)
    torch.testing.assert_close(out[4].view(2, 3), z[4])
    assert gat(h, adj).shape == gat(h.unsqueeze(0), adj.unsqueeze(0))[0].shape


def test_graphsage_aggregators():
    h = torch.arange(12.0).view(4, 3)
    nb = [[1, 2], [0], [], [0, 1, 2]]
    for agg in ("mean", "max"):
        sage = GN.GraphSageLayer(3, 2, aggregator=agg, activation="none")
        a = sage.aggregate(h, nb)
        assert torch.equal(a[2], torch.zeros(3))
        ref = h[[1, 2]].mean(0) if agg == "mean" else h[[1, 2]].max(0).values
        torch.testing.assert_close(a[0], ref)
        assert sage(h, nb).shape == (4, 2)


def test_activity_regularization():
    m = torch.nn.Sequential(torch.nn.Linear(4, 4), R.ActivityRegularization(0.1, 0.01), torch.nn.ReLU(),
                            R.L2ActivityRegularization(0.5))
    x = torch.randn(8, 4)
    y = m(x)
    h = m[0](x)
    want = 0.1 * h.abs().mean() + 0.01 * h.square().mean() + 0.5 * torch.relu(h).square().mean()
    torch.testing.assert_close(R.regularization_loss(m), want)
    assert torch.equal(y, torch.relu(h))
    assert float(R.l2_penalty(m.parameters(), 0.0)) == 0.0


def test_visualization_outputs(tmp_path):
    txt = V.ascii_plot([5, 4, 3, 2.5, 2, 1.8], width=20, height=5, title="loss")
    assert txt.count("*") >= 5 and "loss" in txt
    svg = V.svg_line_plot({"train": [3, 2, 1], "val": [3.5, 2.5, 2]}, str(tmp_path / "c.svg"), "loss")
    assert svg.count("<polyline") == 2 and (tmp_path / "c.svg").exists()
    V.heatmap_svg(torch.rand(4, 4), str(tmp_path / "h.svg"))
    model = torch.nn.Sequential(torch.nn.Conv2d(3, 4, 3), torch.nn.ReLU(), torch.nn.Flatten(),
                                torch.nn.Linear(4 * 6 * 6, 2))
    viz = V.ActivationVisualizer(model)
    model(torch.randn(2, 3, 8, 8))
    st = viz.statistics()
    assert set(st) == {"0", "1", "2", "3"} and st["1"]["min"] >= 0
    assert viz.feature_map("0").shape == (6, 6)
    counts, edges = viz.histogram("3", bins=4)
    assert float(counts.sum()) == 4 and edges.numel() == 5
    s = V.network_summary(model, torch.randn(1, 3, 8, 8))
    assert "Conv2d" in s and "(1, 2)" in s and "total parameters" in s
    w = torch.softmax(torch.randn(1, 3, 5, 5), -1)
    assert V.attention_maps(w).shape == (5, 5) and torch.equal(V.attention_maps(w, heads=1), w[0, 1])
