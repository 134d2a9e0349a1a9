import pytest
import torch

from scirs_b200.metrics import FeatureImportance, LearningCurve


def test_feature_importance_and_learning_curve():
    fi = FeatureImportance(["a", "b", "c"], [0.2, 0.9, 0.5])
    names, vals = fi.top_k(2)
    assert names == ["b", "c"] and torch.allclose(vals, torch.tensor([0.9, 0.5], dtype=torch.float64))
    txt = fi.to_ascii("imp", width=10)
    assert txt.splitlines()[0] == "imp" and txt.splitlines()[1].startswith("b") and "#" * 10 in txt
    with pytest.raises(ValueError):
        FeatureImportance(["a"], [1.0, 2.0])
    lc = LearningCurve([10, 20], [[0.5, 0.7], [0.8, 0.8]], [[0.4, 0.6], [0.7, 0.9]])
    assert torch.allclose(lc.train_mean, torch.tensor([0.6, 0.8], dtype=torch.float64))
    assert torch.allclose(lc.val_std, torch.tensor([0.1, 0.1], dtype=torch.float64))
    assert "validation" in lc.to_ascii("curve")
    with pytest.raises(ValueError):
        LearningCurve([10], [[0.5, 0.7]], [[0.4]])
