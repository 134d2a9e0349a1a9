"""Evaluation metrics (classification, regression, ranking), computed with
tensor ops on the inputs' device.

Reference parity: scirs2-metrics (classification: accuracy, precision,
recall, F1, confusion matrix, ROC curve / AUC, log loss; regression: MSE,
MAE, RMSE, R^2, explained variance) and the neural crate's evaluation
helpers (scirs2-neural/src/utils/evaluation: ROC, confusion matrix).
"""
from __future__ import annotations

import torch


def _labels(pred: torch.Tensor) -> torch.Tensor:
    return pred.argmax(-1) if pred.dim() > 1 and pred.is_floating_point() else pred


def accuracy(pred, target) -> float:
    return float((_labels(pred) == target).float().mean())


def top_k_accuracy(logits, target, k: int = 5) -> float:
    top = logits.topk(k, dim=-1).indices
    return float((top == target.unsqueeze(-1)).any(-1).float().mean())


def confusion_matrix(pred, target, num_classes: int | None = None) -> torch.Tensor:
    p, t = _labels(pred).long().reshape(-1), target.long().reshape(-1)
    n = num_classes or int(max(p.max(), t.max())) + 1
    return torch.bincount(t * n + p, minlength=n * n).reshape(n, n)


def precision_recall_f1(pred, target, num_classes: int | None = None, average: str = "macro"):
    cm = confusion_matrix(pred, target, num_classes).double()
    tp = cm.diag()
    prec = tp / cm.sum(0).clamp(min=1e-12)
    rec = tp / cm.sum(1).clamp(min=1e-12)
    f1 = 2 * prec * rec / (prec + rec).clamp(min=1e-12)
    if average == "macro":
        return float(prec.mean()), float(rec.mean()), float(f1.mean())
    if average == "micro":
        acc = float(tp.sum() / cm.sum())
        return acc, acc, acc
    return prec, rec, f1


def roc_curve(scores, target):
    """Binary ROC: (fpr, tpr, thresholds) with thresholds descending."""
    s, idx = torch.sort(scores.double().reshape(-1), descending=True)
    t = target.reshape(-1)[idx].double()
    tps, fps = torch.cumsum(t, 0), torch.cumsum(1 - t, 0)
    last = torch.cat([s[1:] != s[:-1], torch.tensor([True], device=s.device)])
    tps, fps, thr = tps[last], fps[last], s[last]
    zero = torch.zeros(1, dtype=torch.float64, device=s.device)
    tpr = torch.cat([zero, tps / tps[-1].clamp(min=1)])
    fpr = torch.cat([zero, fps / fps[-1].clamp(min=1)])
    return fpr, tpr, torch.cat([torch.full((1,), float("inf"), dtype=torch.float64, device=s.device), thr])


def roc_auc(scores, target) -> float:
    fpr, tpr, _ = roc_curve(scores, target)
    return float(torch.trapz(tpr, fpr))


def log_loss(probs, target, eps: float = 1e-15) -> float:
    p = probs.double().clamp(eps, 1 - eps)
    if p.dim() == 1:
        t = target.double()
        return float(-(t * p.log() + (1 - t) * (1 - p).log()).mean())
    return float(-p.gather(-1, target.long().unsqueeze(-1)).log().mean())


def mse(pred, target) -> float:
    return float(((pred.double() - target.double()) ** 2).mean())


def rmse(pred, target) -> float:
    return mse(pred, target) ** 0.5


def mae(pred, target) -> float:
    return float((pred.double() - target.double()).abs().mean())


def r2_score(pred, target) -> float:
    t = target.double()
    ss_res = ((t - pred.double()) ** 2).sum()
    ss_tot = ((t - t.mean()) ** 2).sum()
    return float(1 - ss_res / ss_tot.clamp(min=1e-300))


def explained_variance(pred, target) -> float:
    t, p = target.double(), pred.double()
    return float(1 - (t - p).var(unbiased=False) / t.var(unbiased=False).clamp(min=1e-300))


def perplexity(mean_nll: float) -> float:
    import math

    return math.exp(mean_nll)


# ---------------------------------------------------------------------------- evaluation summaries
class FeatureImportance:
    """Named importance scores with a top-k selection and a text bar chart.
    Reference parity: scirs2-neural/src/utils/evaluation/feature_importance.rs:20-160."""

    def __init__(self, feature_names: list, importance):
        imp = torch.as_tensor(importance, dtype=torch.float64).reshape(-1)
        if len(feature_names) != imp.numel():
            raise ValueError("Number of feature names must match number of importance scores")
        self.feature_names, self.importance = list(feature_names), imp

    def top_k(self, k: int):
        k = min(int(k), len(self.feature_names))
        order = torch.argsort(self.importance, descending=True, stable=True)[:k]
        return [self.feature_names[i] for i in order.tolist()], self.importance[order]

    def to_ascii(self, title: str | None = None, width: int = 40, k: int | None = None) -> str:
        names, vals = self.top_k(k if k is not None else len(self.feature_names))
        top = float(vals.abs().max()) if vals.numel() else 0.0
        pad = max((len(n) for n in names), default=0)
        lines = [title] if title else []
        for n, v in zip(names, vals.tolist()):
            bar = "#" * (int(round(abs(v) / top * width)) if top > 0 else 0)
            lines.append(f"{n.ljust(pad)} | {bar} {v:.4f}")
        return "\n".join(lines)


class LearningCurve:
    """Scores [n_sizes, n_folds] for the training and validation sets at each training size, with
    per-size means and (population) standard deviations over the folds.
    Reference parity: scirs2-neural/src/utils/evaluation/learning_curve.rs:19-160."""

    def __init__(self, train_sizes, train_scores, val_scores):
        self.train_sizes = [int(s) for s in train_sizes]
        tr = torch.as_tensor(train_scores, dtype=torch.float64)
        va = torch.as_tensor(val_scores, dtype=torch.float64)
        if tr.dim() != 2 or va.dim() != 2 or tr.shape[0] != len(self.train_sizes) or va.shape[0] != len(self.train_sizes):
            raise ValueError("Number of scores must match number of training sizes")
        if tr.shape[1] != va.shape[1]:
            raise ValueError("Training and validation scores must have the same number of CV folds")
        self.train_scores, self.val_scores = tr, va
        self.train_mean, self.val_mean = tr.mean(1), va.mean(1)
        self.train_std, self.val_std = tr.std(1, unbiased=False), va.std(1, unbiased=False)

    def to_ascii(self, title: str | None = None, width: int = 50, height: int = 12) -> str:
        from .utils.visualization import ascii_plot

        head = (title + "\n") if title else ""
        return (head + "train\n" + ascii_plot(self.train_mean.tolist(), width, height)
                + "\nvalidation\n" + ascii_plot(self.val_mean.tolist(), width, height))
