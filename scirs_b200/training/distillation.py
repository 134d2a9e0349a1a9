"""Knowledge distillation losses and trainer.

Methods: response-based (temperature-softened KL between teacher and student
logits, mixed with the hard-label loss: alpha * T^2 * KL + beta * CE),
feature-based (student features adapted by a linear map, MSE to the teacher
features), attention-based (spatial / channel attention maps, L2 between
normalised maps), relation-based (pairwise sample distance matrices) and
self-distillation from an ensemble of the student's own snapshots.

Reference parity: scirs2-neural/src/distillation.rs:20-860
(DistillationMethod, FeatureAdaptation, AttentionType, RelationType,
DistanceMetric, EnsembleAggregation, DistillationTrainer,
compute_distillation_loss, statistics).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F


class DistanceMetric(enum.Enum):
    EUCLIDEAN = "euclidean"
    COSINE = "cosine"
    MANHATTAN = "manhattan"
    KL_DIVERGENCE = "kl"


class AttentionType(enum.Enum):
    SPATIAL = "spatial"
    CHANNEL = "channel"


class EnsembleAggregation(enum.Enum):
    AVERAGE = "average"
    SOFT_VOTING = "soft_voting"


def response_loss(student_logits, teacher_logits, targets=None, temperature: float = 4.0, alpha: float = 0.7,
                  beta: float = 0.3):
    t = temperature
    kl = F.kl_div(F.log_softmax(student_logits / t, -1), F.softmax(teacher_logits.detach() / t, -1),
                  reduction="batchmean") * (t * t)
    loss = alpha * kl
    if targets is not None and beta:
        loss = loss + beta * F.cross_entropy(student_logits, targets)
    return loss


def attention_map(feat: torch.Tensor, kind: AttentionType = AttentionType.SPATIAL) -> torch.Tensor:
    """feat [N, C, H, W] -> L2-normalised attention map."""
    if kind == AttentionType.SPATIAL:
        a = feat.pow(2).mean(1).flatten(1)
    else:
        a = feat.pow(2).mean((2, 3))
    return F.normalize(a, dim=1)


def pairwise_distance(x: torch.Tensor, metric: DistanceMetric) -> torch.Tensor:
    x = x.flatten(1)
    if metric == DistanceMetric.EUCLIDEAN:
        d = torch.cdist(x, x)
    elif metric == DistanceMetric.MANHATTAN:
        d = torch.cdist(x, x, p=1)
    elif metric == DistanceMetric.COSINE:
        n = F.normalize(x, dim=1)
        d = 1 - n @ n.t()
    else:
        p = F.softmax(x, -1)
        lp = F.log_softmax(x, -1)
        d = (p[:, None, :] * (lp[:, None, :] - lp[None, :, :])).sum(-1)
    return d / d.mean().clamp(min=1e-12)


def relation_loss(student_feat, teacher_feat, metric: DistanceMetric = DistanceMetric.EUCLIDEAN):
    return F.smooth_l1_loss(pairwise_distance(student_feat, metric), pairwise_distance(teacher_feat.detach(), metric))


@dataclass
class DistillationConfig:
    method: str = "response"  # response | feature | attention | relation | self
    temperature: float = 4.0
    alpha: float = 0.7
    beta: float = 0.3
    feature_weight: float = 1.0
    distance: DistanceMetric = DistanceMetric.EUCLIDEAN
    attention: AttentionType = AttentionType.SPATIAL
    ensemble_size: int = 3


@dataclass
class DistillationStatistics:
    steps: int = 0
    distill_loss: list = field(default_factory=list)
    hard_loss: list = field(default_factory=list)


class DistillationTrainer:
    """Trains `student` to match `teacher`. For feature/attention/relation
    methods the models must return (logits, features)."""

    def __init__(self, student: nn.Module, teacher: nn.Module, config: DistillationConfig | None = None,
                 optimizer=None):
        self.student, self.teacher = student, teacher
        self.config = config or DistillationConfig()
        self.opt = optimizer or torch.optim.Adam(student.parameters(), lr=1e-3)
        self.adapters: dict[str, nn.Module] = {}
        self.stats = DistillationStatistics()
        self._snapshots: list = []
        teacher.eval()

    def add_adaptation_layer(self, name: str, s_dim: int, t_dim: int):
        layer = nn.Linear(s_dim, t_dim, bias=False)
        self.adapters[name] = layer
        self.opt.add_param_group({"params": layer.parameters()})
        return layer

    def compute_distillation_loss(self, x, y):
        c = self.config
        with torch.no_grad():
            t_out = self.teacher(x)
        s_out = self.student(x)
        s_logits, s_feat = (s_out if isinstance(s_out, tuple) else (s_out, None))
        t_logits, t_feat = (t_out if isinstance(t_out, tuple) else (t_out, None))
        hard = F.cross_entropy(s_logits, y)
        if c.method == "response":
            dl = response_loss(s_logits, t_logits, None, c.temperature, c.alpha, 0.0)
            return dl + c.beta * hard, dl, hard
        if c.method == "feature":
            sf = s_feat.flatten(1)
            ad = self.adapters.get("feature") or self.add_adaptation_layer("feature", sf.shape[1],
                                                                          t_feat.flatten(1).shape[1])
            dl = c.feature_weight * F.mse_loss(ad(sf), t_feat.flatten(1).detach())
        elif c.method == "attention":
            dl = c.feature_weight * (attention_map(s_feat, c.attention) - attention_map(t_feat, c.attention).detach()
                                     ).pow(2).sum(1).mean()
        elif c.method == "relation":
            dl = c.feature_weight * relation_loss(s_feat, t_feat, c.distance)
        elif c.method == "self":
            if not self._snapshots:
                return hard, hard.detach() * 0, hard
            with torch.no_grad():
                ens = torch.stack([F.softmax(m(x)[0] if isinstance(m(x), tuple) else m(x), -1)
                                   for m in self._snapshots]).mean(0)
            dl = F.kl_div(F.log_softmax(s_logits, -1), ens, reduction="batchmean")
        else:
            raise ValueError(c.method)
        return dl + c.beta * hard, dl, hard

    def train_step(self, x, y) -> float:
        self.student.train()
        loss, dl, hard = self.compute_distillation_loss(x, y)
        self.opt.zero_grad()
        loss.backward()
        self.opt.step()
        self.stats.steps += 1
        self.stats.distill_loss.append(float(dl))
        self.stats.hard_loss.append(float(hard))
        return float(loss)

    def snapshot(self):
        """Add a frozen copy of the student to the self-distillation ensemble."""
        import copy

        m = copy.deepcopy(self.student).eval()
        self._snapshots = (self._snapshots + [m])[-self.config.ensemble_size:]

    def get_statistics(self) -> DistillationStatistics:
        return self.stats

    def reset_statistics(self):
        self.stats = DistillationStatistics()
