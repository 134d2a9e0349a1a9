"""Distillation, federated averaging and gradient compression."""
import torch
import torch.nn as nn

from scirs_b200.parallel.compression import (OneBitQuantizer, TopKCompressor, TopKConfig, low_rank_compress,
                                             low_rank_decompress)
from scirs_b200.training.distillation import DistillationConfig, DistillationTrainer, response_loss
from scirs_b200.training.federated import (AggregationMethod, ClientUpdate, FederatedConfig, FederatedServer)


def test_response_distillation_transfers_teacher():
    torch.manual_seed(0)
    teacher = nn.Sequential(nn.Linear(6, 32), nn.ReLU(), nn.Linear(32, 3))
    student = nn.Linear(6, 3)
    x = torch.randn(256, 6)
    y = teacher(x).argmax(-1)
    tr = DistillationTrainer(student, teacher, DistillationConfig(temperature=2.0, alpha=1.0, beta=0.1),
                             torch.optim.Adam(student.parameters(), lr=0.05))
    for _ in range(150):
        tr.train_step(x, y)
    agree = float((student(x).argmax(-1) == y).float().mean())
    assert agree > 0.8 and tr.get_statistics().steps == 150
    assert float(response_loss(teacher(x), teacher(x), None, 2.0, 1.0, 0.0)) < 1e-5


def test_feature_and_relation_distillation_run():
    torch.manual_seed(1)

    class Net(nn.Module):
        def __init__(self, w):
            super().__init__()
            self.f = nn.Linear(4, w)
            self.h = nn.Linear(w, 2)

        def forward(self, x):
            z = torch.relu(self.f(x))
            return self.h(z), z

    x, y = torch.randn(32, 4), torch.randint(0, 2, (32,))
    for method in ("feature", "relation", "self"):
        tr = DistillationTrainer(Net(8), Net(16), DistillationConfig(method=method))
        if method == "self":
            tr.snapshot()
        losses = [tr.train_step(x, y) for _ in range(5)]
        assert all(l == l for l in losses)


def test_federated_fedavg_and_median():
    cfg = FederatedConfig.builder().num_rounds(2).clients_per_round(3).seed(0).build()
    srv = FederatedServer(cfg, [torch.zeros(4)])
    ups = [ClientUpdate(i, [torch.full((4,), float(i + 1))], num_samples=n).with_loss(1.0)
           for i, n in enumerate([1, 1, 2])]
    st = srv.aggregate(ups)
    assert torch.allclose(srv.global_params()[0], torch.full((4,), (1 + 2 + 6) / 4.0))
    assert st.num_clients == 3 and not srv.is_complete()
    cfg2 = FederatedConfig(aggregation=AggregationMethod.MEDIAN, clients_per_round=3)
    srv2 = FederatedServer(cfg2, [torch.zeros(2)])
    srv2.aggregate([ClientUpdate(i, [torch.full((2,), v)], 1) for i, v in enumerate([1.0, 100.0, 2.0])])
    assert torch.allclose(srv2.global_params()[0], torch.full((2,), 2.0))
    assert len(srv.select_clients(10)) == 3
    dp = FederatedConfig.builder().differential_privacy(1.0, 0.5).build()
    s3 = FederatedServer(dp, [torch.zeros(3)])
    assert s3.aggregate([ClientUpdate(0, [torch.ones(3) * 10], 1)]).epsilon > 0


def test_gradient_compression():
    g = torch.randn(1000)
    c = TopKCompressor(1000, TopKConfig(0.1))
    idx, vals = c.compress(g)
    rec = TopKCompressor.decompress(idx, vals, 1000)
    assert idx.numel() == 100 and torch.allclose(rec + c.residual, g)
    bits, scale = OneBitQuantizer.quantize(g)
    q = OneBitQuantizer.dequantize(bits, scale, 1000)
    assert OneBitQuantizer.quantization_error(g, q) < 1.0
    m = torch.randn(64, 8) @ torch.randn(8, 32)
    p, qq = low_rank_compress(m, rank=8)
    assert torch.allclose(low_rank_decompress(p, qq), m, atol=1e-3)
