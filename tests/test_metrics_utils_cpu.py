"""Metrics, profiling helpers and configuration."""
import torch

from scirs_b200 import metrics as M
from scirs_b200.utils.profiling import Config, Metrics, Profiler, Timer


def test_classification_metrics():
    logits = torch.tensor([[2.0, 0.1, 0.0], [0.1, 3.0, 0.2], [0.0, 0.1, 1.0], [1.0, 0.0, 0.5]])
    y = torch.tensor([0, 1, 2, 2])
    assert M.accuracy(logits, y) == 0.75
    cm = M.confusion_matrix(logits, y, 3)
    assert cm.tolist() == [[1, 0, 0], [0, 1, 0], [1, 0, 1]]
    p, r, f = M.precision_recall_f1(logits, y, 3)
    assert abs(r - (1 + 1 + 0.5) / 3) < 1e-9 and 0 < f <= 1
    assert M.top_k_accuracy(logits, y, 2) == 1.0


def test_roc_auc_and_regression():
    s = torch.tensor([0.1, 0.4, 0.35, 0.8])
    t = torch.tensor([0, 0, 1, 1])
    assert abs(M.roc_auc(s, t) - 0.75) < 1e-12
    x = torch.tensor([1.0, 2.0, 3.0])
    assert M.mse(x, x) == 0.0 and M.r2_score(x, x) == 1.0 and abs(M.mae(x + 1, x) - 1) < 1e-12
    assert abs(M.log_loss(torch.tensor([0.9, 0.1]), torch.tensor([1, 0])) + torch.log(torch.tensor(0.9)).item()) < 1e-6


def test_profiler_metrics_config():
    prof = Profiler()
    with prof.section("a"):
        pass
    with Timer() as t:
        pass
    assert prof.calls["a"] == 1 and "a" in prof.report() and t.elapsed >= 0
    m = Metrics()
    m.inc("steps", labels={"rank": 0})
    m.set("lr", 0.1)
    m.observe("latency", 0.05)
    txt = m.prometheus_text()
    assert 'steps_total{rank="0"} 1.0' in txt and "latency_count 1" in txt
    c = Config({"SCIRS_THREADS": "8", "SCIRS_FAST": "yes", "OTHER": "x"})
    assert c.get_int("threads") == 8 and c.get_bool("fast") and c.keys() == ["threads", "fast"]
