"""Loss functions (scirs2-neural/src/losses/*.rs).

`CrossEntropyLoss` accepts either logits + integer class indices (the
Python API contract, scirs2-python/tests/test_neural.py:240-246; bf16 CUDA
logits run on the fused softmax-cross-entropy kernel) or, with
`from_logits=False`, probabilities + one-hot / soft targets, which is the
reference Rust semantics (losses/crossentropy.rs:54-143: loss = -sum t log p / N,
gradient (p - t) / N).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import functional as FN


class Loss:
    def forward(self, predictions, targets) -> torch.Tensor:
        raise NotImplementedError

    def __call__(self, predictions, targets):
        return self.forward(predictions, targets)

    def backward(self, predictions, targets) -> torch.Tensor:
        """d loss / d predictions (reference Loss::backward)."""
        p = predictions.detach().requires_grad_(True)
        with torch.enable_grad():
            loss = self.forward(p, targets)
        (g,) = torch.autograd.grad(loss, p)
        return g


class MSELoss(Loss):
    def forward(self, p, t):
        return F.mse_loss(p, t.to(p.dtype))


class MAELoss(Loss):
    def forward(self, p, t):
        return F.l1_loss(p, t.to(p.dtype))


class HuberLoss(Loss):
    def __init__(self, delta: float = 1.0):
        self.delta = delta

    def forward(self, p, t):
        return F.huber_loss(p, t.to(p.dtype), delta=self.delta)


class CrossEntropyLoss(Loss):
    def __init__(self, from_logits: bool = True, ignore_index: int = -100, epsilon: float = 1e-10):
        self.from_logits, self.ignore_index, self.eps = from_logits, ignore_index, epsilon

    def forward(self, p, t):
        if not self.from_logits:
            return -(t.to(p.dtype) * torch.log(p.clamp(min=self.eps))).sum() / p.shape[0]
        if t.dtype in (torch.int64, torch.int32, torch.int16, torch.uint8):
            logits = p.reshape(-1, p.shape[-1])
            return FN.cross_entropy(logits, t.reshape(-1), self.ignore_index)
        return torch.sum(-t * F.log_softmax(p.float(), -1)) / p.shape[0]


class BinaryCrossEntropyLoss(Loss):
    def __init__(self, from_logits: bool = False):
        self.from_logits = from_logits

    def forward(self, p, t):
        t = t.to(p.dtype)
        if self.from_logits:
            return F.binary_cross_entropy_with_logits(p, t)
        return F.binary_cross_entropy(p.clamp(1e-7, 1 - 1e-7), t)


class FocalLoss(Loss):
    """Multi-class focal loss on logits: -alpha (1-p_t)^gamma log p_t."""

    def __init__(self, gamma: float = 2.0, alpha: float = 0.25):
        self.gamma, self.alpha = gamma, alpha

    def forward(self, p, t):
        logp = F.log_softmax(p.float(), -1)
        lpt = logp.gather(-1, t.long().unsqueeze(-1)).squeeze(-1)
        return (-self.alpha * (1 - lpt.exp()) ** self.gamma * lpt).mean()


class ContrastiveLoss(Loss):
    """Pairs (x1, x2) with label 1 = similar: y d^2 + (1-y) max(0, m - d)^2."""

    def __init__(self, margin: float = 1.0):
        self.margin = margin

    def forward(self, pair, y):
        x1, x2 = pair
        d = F.pairwise_distance(x1, x2)
        y = y.to(d.dtype)
        return (y * d**2 + (1 - y) * torch.clamp(self.margin - d, min=0) ** 2).mean() / 2


class TripletLoss(Loss):
    def __init__(self, margin: float = 1.0):
        self.margin = margin

    def forward(self, triple, _unused=None):
        a, pos, neg = triple
        return F.triplet_margin_loss(a, pos, neg, margin=self.margin)


class KLDivLoss(Loss):
    def forward(self, log_p, q):
        return F.kl_div(log_p, q, reduction="batchmean")


# ---------------------------------------------------------------------------- functional forms
# Binary / segmentation and metric-learning losses on probabilities and embeddings, differentiable
# (scirs2-neural/src/losses/extended.rs:52-330: focal_loss, dice_loss, tversky_loss,
# contrastive_loss, triplet_loss; the same definitions and smoothing constants).


def _same_shape(a, b, what):
    if a.shape != b.shape:
        raise ValueError(f"{what}: shape mismatch {tuple(a.shape)} vs {tuple(b.shape)}")
    if a.numel() == 0:
        raise ValueError(f"{what}: empty tensors")


def focal_loss(preds, targets, alpha: float = 0.25, gamma: float = 2.0):
    """Binary focal loss on probabilities: mean of -alpha_t (1 - p_t)^gamma log p_t, with
    p_t = p for targets > 0.5 (else 1 - p), alpha_t = alpha (else 1 - alpha), p clamped to
    [1e-12, 1 - 1e-12]."""
    _same_shape(preds, targets, "focal_loss")
    p = preds.clamp(1e-12, 1 - 1e-12)
    pos = targets > 0.5
    pt = torch.where(pos, p, 1 - p)
    at = torch.where(pos, torch.full_like(p, alpha), torch.full_like(p, 1 - alpha))
    return (-at * (1 - pt) ** gamma * pt.log()).mean()


def dice_loss(preds, targets):
    """1 - (2 sum(p t) + eps) / (sum p + sum t + eps), eps = 1e-8."""
    _same_shape(preds, targets, "dice_loss")
    eps = 1e-8
    return 1 - (2 * (preds * targets).sum() + eps) / (preds.sum() + targets.sum() + eps)


def tversky_loss(preds, targets, alpha: float = 0.5, beta: float = 0.5):
    """1 - (TP + eps) / (TP + alpha FP + beta FN + eps) with soft counts TP = sum p t,
    FP = sum p (1 - t), FN = sum (1 - p) t; alpha = beta = 0.5 is the dice loss."""
    _same_shape(preds, targets, "tversky_loss")
    eps = 1e-8
    tp = (preds * targets).sum()
    fp = (preds * (1 - targets)).sum()
    fn = ((1 - preds) * targets).sum()
    return 1 - (tp + eps) / (tp + alpha * fp + beta * fn + eps)


def contrastive_loss(e1, e2, labels, margin: float = 1.0):
    """mean over pairs of y d^2 + (1 - y) max(0, margin - d)^2, d the Euclidean distance of the
    [batch, dim] embeddings (labels 1 = similar)."""
    if e1.dim() != 2 or e1.shape != e2.shape or labels.shape != (e1.shape[0],):
        raise ValueError("contrastive_loss: embeddings must be matching [batch, dim], labels [batch]")
    d2 = ((e1 - e2) ** 2).sum(1)
    d = d2.sqrt()
    y = labels.to(d.dtype)
    return (y * d2 + (1 - y) * torch.clamp(margin - d, min=0) ** 2).mean()


def triplet_loss(anchor, positive, negative, margin: float = 1.0):
    """mean of max(0, |a - p|^2 - |a - n|^2 + margin) over [batch, dim] triplets (squared distances)."""
    if anchor.dim() != 2 or anchor.shape != positive.shape or anchor.shape != negative.shape:
        raise ValueError("triplet_loss: inputs must be matching [batch, dim]")
    dap = ((anchor - positive) ** 2).sum(1)
    dan = ((anchor - negative) ** 2).sum(1)
    return torch.clamp(dap - dan + margin, min=0).mean()


class DiceLoss(Loss):
    def forward(self, p, t):
        return dice_loss(p, t)


class TverskyLoss(Loss):
    def __init__(self, alpha: float = 0.5, beta: float = 0.5):
        self.alpha, self.beta = alpha, beta

    def forward(self, p, t):
        return tversky_loss(p, t, self.alpha, self.beta)


def get_loss(name) -> Loss:
    if isinstance(name, Loss):
        return name
    n = str(name).lower()
    table = {
        "mse": MSELoss, "mean_squared_error": MSELoss, "mae": MAELoss, "huber": HuberLoss,
        "crossentropy": CrossEntropyLoss, "cross_entropy": CrossEntropyLoss, "categorical_crossentropy": CrossEntropyLoss,
        "bce": BinaryCrossEntropyLoss, "binary_crossentropy": BinaryCrossEntropyLoss, "focal": FocalLoss,
        "dice": DiceLoss, "tversky": TverskyLoss, "kl_div": KLDivLoss,
    }
    if n not in table:
        raise ValueError(f"unknown loss {name}")
    return table[n]()
