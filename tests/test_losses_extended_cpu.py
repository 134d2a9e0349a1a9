"""Functional binary / segmentation / metric-learning losses against
restatements of their definitions (float64), with gradients by autograd."""
import math

import pytest
import torch

from scirs_b200.nn import losses as L


def test_focal_matches_definition_and_doc_example():
    p = torch.tensor([0.9, 0.6, 0.2, 0.1], dtype=torch.float64)
    t = torch.tensor([1.0, 1.0, 0.0, 0.0], dtype=torch.float64)
    ref = 0.0
    for pi, ti in zip(p.tolist(), t.tolist()):
        pt = pi if ti > 0.5 else 1 - pi
        at = 0.25 if ti > 0.5 else 0.75
        ref += -at * (1 - pt) ** 2 * math.log(pt)
    assert L.focal_loss(p, t, 0.25, 2.0).item() == pytest.approx(ref / 4, rel=1e-12)


def test_dice_and_tversky():
    p = torch.tensor([0.9, 0.1, 0.8, 0.3], dtype=torch.float64, requires_grad=True)
    t = torch.tensor([1.0, 0.0, 1.0, 1.0], dtype=torch.float64)
    inter, sp, st = 0.9 + 0.8 + 0.3, 2.1, 3.0
    assert L.dice_loss(p, t).item() == pytest.approx(1 - (2 * inter + 1e-8) / (sp + st + 1e-8), rel=1e-12)
    assert L.tversky_loss(p, t, 0.5, 0.5).item() == pytest.approx(L.dice_loss(p, t).item(), abs=1e-7)  # eps placement
    tp, fp, fn = inter, 0.1, 0.1 + 0.2 + 0.7
    assert L.tversky_loss(p, t, 0.3, 0.7).item() == pytest.approx(1 - (tp + 1e-8) / (tp + 0.3 * fp + 0.7 * fn + 1e-8))
    L.DiceLoss()(p, t).backward()
    assert p.grad is not None and torch.isfinite(p.grad).all()
    assert isinstance(L.get_loss("tversky"), L.TverskyLoss)
    with pytest.raises(ValueError):
        L.dice_loss(p, t[:3])


def test_contrastive_and_triplet():
    g = torch.Generator().manual_seed(0)
    e1, e2 = torch.randn(5, 3, generator=g, dtype=torch.float64), torch.randn(5, 3, generator=g, dtype=torch.float64)
    y = torch.tensor([1, 0, 1, 0, 0])
    ref = 0.0
    for i in range(5):
        d = (e1[i] - e2[i]).norm().item()
        ref += d * d if y[i] else max(0.0, 1.5 - d) ** 2
    assert L.contrastive_loss(e1, e2, y, 1.5).item() == pytest.approx(ref / 5, rel=1e-12)
    a, pos, neg = (torch.randn(4, 6, generator=g, dtype=torch.float64) for _ in range(3))
    ref = sum(max(0.0, ((a[i] - pos[i]) ** 2).sum().item() - ((a[i] - neg[i]) ** 2).sum().item() + 0.5)
              for i in range(4)) / 4
    assert L.triplet_loss(a, pos, neg, 0.5).item() == pytest.approx(ref, rel=1e-12)
    with pytest.raises(ValueError):
        L.triplet_loss(a, pos, neg[:, :2])
