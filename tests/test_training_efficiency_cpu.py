"""Activation checkpoint manager / recomputation, sparse training, progress monitor (CPU)."""
import io

import torch
import torch.nn as nn

from scirs_b200.training import efficiency as E


def test_manager_policies_budget_and_eviction():
    m = E.GradientCheckpointManager(100, E.RecomputationPolicy.checkpoint_all())
    a = torch.zeros(10, dtype=torch.float32)  # 40 bytes
    assert m.checkpoint_activation(0, a, 1) and m.checkpoint_activation(1, a, 1)
    assert m.memory_usage() == 80 and m.num_checkpoints() == 2
    assert m.checkpoint_activation(2, a, 1)  # evicts layer 0
    assert not m.has_checkpoint(0) and m.has_checkpoint(1) and m.has_checkpoint(2)
    st = m.get_statistics()
    assert st.total_checkpoints == 3 and st.in_memory_checkpoints == 2 and st.total_memory == 80
    assert abs(st.memory_utilization - 0.8) < 1e-12
    t = m.get_checkpoint(1)
    assert torch.equal(t, a) and not m.has_checkpoint(1) and m.memory_usage() == 40
    m.clear()
    assert m.num_checkpoints() == 0 and m.memory_usage() == 0
    assert not E.GradientCheckpointManager(100, E.RecomputationPolicy.checkpoint_none()).checkpoint_activation(0, a, 9)
    sel = E.GradientCheckpointManager(1000, E.RecomputationPolicy.selective(50))
    assert not sel.checkpoint_activation(0, a, 10) and sel.checkpoint_activation(1, a, 60)
    ev = E.GradientCheckpointManager(1000, E.RecomputationPolicy.every_n(2))
    assert ev.checkpoint_activation(4, a, 0) and not ev.checkpoint_activation(3, a, 0)


def test_recomputation_gives_identical_gradients():
    torch.manual_seed(0)
    net = nn.Sequential(nn.Linear(8, 16), nn.Tanh(), nn.Linear(16, 4))
    x = torch.randn(5, 8)
    ref = net(x).pow(2).sum()
    ref.backward()
    g_ref = [p.grad.clone() for p in net.parameters()]
    net.zero_grad()
    eb = E.EfficientBackprop(10_000, E.RecomputationPolicy.checkpoint_none())
    h = eb.forward_with_checkpoint(0, x, net[0], 1)
    h = eb.forward_with_checkpoint(1, h, net[1], 1)
    y = eb.forward_with_checkpoint(2, h, net[2], 1)
    y.pow(2).sum().backward()
    assert eb.recomputed_bytes > 0
    assert all(torch.allclose(p.grad, g) for p, g in zip(net.parameters(), g_ref))


def test_sparse_training_and_progress_monitor():
    torch.manual_seed(1)
    net = nn.Sequential(nn.Linear(10, 10), nn.ReLU(), nn.Linear(10, 2))
    sp = E.SparseTraining(net, E.SparseTrainingConfig(enabled=True, sparsity_ratio=0.5))
    assert abs(sp.sparsity() - 0.5) < 0.06
    opt = torch.optim.SGD(net.parameters(), lr=0.1)
    net(torch.randn(4, 10)).sum().backward()
    opt.step()
    sp.apply()
    assert float((net[0].weight == 0).float().mean()) >= 0.45
    buf = io.StringIO()
    pm = E.ProgressMonitor(E.ProgressMonitorConfig(update_frequency=2), stream=buf)
    for s in range(5):
        pm.on_batch_end(s, None, {"loss": 0.5})
    assert pm.reports == ["step 2: loss=0.5", "step 4: loss=0.5"] and "step 4" in buf.getvalue()
