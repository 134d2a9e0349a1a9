"""AdaLoRA, bottleneck adapters and LoRA merge / int8 utilities (CPU, float64)."""
import math

import pytest
import torch

from scirs_b200.nn import lora as L


def test_adalora_forward_importance_and_pruning():
    torch.manual_seed(0)
    W = torch.randn(6, 5, dtype=torch.float64)
    layer = L.AdaLoRALinear(W, L.AdaLoraConfig(initial_rank=4, target_rank=2, alpha=2.0))
    x = torch.randn(3, 5, dtype=torch.float64)
    assert torch.allclose(layer(x), x @ W.t())  # s = 0: W_eff = W
    with torch.no_grad():
        layer.singular_values.copy_(torch.tensor([1.0, -2.0, 0.5, 3.0], dtype=torch.float64))
    lam = layer.singular_values * (2.0 / 4)
    weff = W + layer.u_mat @ torch.diag(lam) @ layer.v_mat
    assert torch.allclose(layer.effective_weight(), weff)
    assert torch.allclose(layer(x), x @ weff.t())
    loss = (layer(x) ** 2).sum()
    loss.backward()
    assert layer.u_mat.grad is not None and layer.v_mat.grad is not None and layer.weight.grad is None
    layer.update_importance()
    sens = (layer.singular_values * layer.singular_values.grad).abs().float()
    assert torch.allclose(layer.importance_ema, 0.15 * sens)
    keep = layer.prune_to_budget(2)
    assert keep == 2 and layer.active_rank() == 2
    top = torch.argsort(sens, descending=True)[:2]
    assert set(torch.nonzero(layer.rank_mask).flatten().tolist()) == set(top.tolist())
    mask = layer.rank_mask
    assert torch.allclose(layer.effective_weight(), W + layer.u_mat @ torch.diag(lam * mask) @ layer.v_mat)
    assert layer.budget_at(5, 100) == 4 and layer.budget_at(100, 100) == 2
    assert 2 <= layer.budget_at(50, 100) <= 4
    assert float(layer.orthogonality_penalty()) >= 0
    with pytest.raises(ValueError):
        L.AdaLoRALinear(W, L.AdaLoraConfig(initial_rank=2, target_rank=3))
    with pytest.raises(ValueError):
        layer.update_importance(torch.zeros(3))


def test_bottleneck_adapter():
    a = L.BottleneckAdapter(8, L.AdapterConfig(bottleneck_dim=3, activation="gelu", seed=7), dtype=torch.float64)
    b = L.BottleneckAdapter(8, L.AdapterConfig(bottleneck_dim=3, activation="gelu", seed=7), dtype=torch.float64)
    assert torch.equal(a.down_project, b.down_project) and torch.equal(a.up_project, b.up_project)
    bound = math.sqrt(6.0 / 11)
    assert float(a.down_project.abs().max()) <= bound and float(a.up_project.abs().max()) <= bound
    x = torch.randn(4, 8, dtype=torch.float64)
    h = x @ a.down_project.t()
    g = 0.5 * h * (1 + torch.tanh(math.sqrt(2 / math.pi) * (h + 0.044715 * h ** 3)))
    assert torch.allclose(a(x), x + g @ a.up_project.t())
    c = L.BottleneckAdapter(8, L.AdapterConfig(bottleneck_dim=3, activation="relu", residual=False),
                            dtype=torch.float64)
    assert torch.allclose(c(x), torch.relu(x @ c.down_project.t()) @ c.up_project.t())
    assert a.stats()["trainable_params"] == 2 * 3 * 8 + 3 + 8
    with pytest.raises(ValueError):
        L.AdapterConfig(bottleneck_dim=0).validate()
    with pytest.raises(ValueError):
        a(torch.randn(2, 5, dtype=torch.float64))


def test_merge_and_quantize():
    W = torch.eye(4, dtype=torch.float64)
    A = torch.arange(8, dtype=torch.float64).view(2, 4) * 0.1
    B = torch.arange(8, dtype=torch.float64).view(4, 2) * 0.1
    m = L.merge_lora_weights(W, A, B, 0.5)
    assert torch.allclose(m, W + 0.5 * B @ A)
    with pytest.raises(ValueError):
        L.merge_lora_weights(W, torch.zeros(2, 3), B, 1.0)
    m2 = L.merge_multiple_lora(W, [(A, B, 0.5), (A, B, 0.25)])
    assert torch.allclose(m2, W + 0.75 * B @ A)
    q = L.quantize_merged_weight(m2)
    assert q.data.dtype == torch.int8 and q.rows == 4 and q.cols == 4 and q.compression_ratio() == 8.0
    assert abs(q.scale - float(m2.abs().max()) / 127) < 1e-15
    assert q.quantization_error(m2) <= q.scale / 2 + 1e-12
    z = L.quantize_merged_weight(torch.zeros(2, 2))
    assert z.scale == 1.0 and int(z.data.abs().sum()) == 0
    with pytest.raises(ValueError):
        L.quantize_merged_weight(m2, bits=4)
    lora = L.LoRALinear(torch.randn(5, 6, dtype=torch.float64), L.LoRAConfig(rank=2, alpha=4.0))
    with torch.no_grad():
        lora.lora_b.normal_()
    eff = L.compute_effective_weight(lora)
    lora.merge()
    assert torch.allclose(L.compute_effective_weight(lora), eff)
