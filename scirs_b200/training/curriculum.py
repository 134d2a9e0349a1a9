"""Curriculum learning: which samples an epoch trains on.

competence(t) grows from `initial_competence` to 1 (linear, sqrt, or in
`num_steps` steps) over `num_epochs`; BabyStep (and AntiCurriculum, on the
reversed difficulty order) uses the easiest ceil(c*N) samples, OnePass only
the band unlocked since the previous epoch, SelfPaced the samples whose last
loss is below a threshold that grows by `self_paced_growth_rate` per loss
update (topped up with the easiest samples to `min_samples`).

Reference parity: scirs2-neural/src/training/curriculum.rs:60-700.
"""
from __future__ import annotations

import enum
import math
import random
from dataclasses import dataclass


class CurriculumStrategy(enum.Enum):
    BABY_STEP = "baby_step"
    ONE_PASS = "one_pass"
    SELF_PACED = "self_paced"
    ANTI_CURRICULUM = "anti_curriculum"


@dataclass
class CompetenceSchedule:
    kind: str = "linear"  # "linear" | "sqrt" | "step"
    num_steps: int = 1


@dataclass
class CurriculumConfig:
    strategy: CurriculumStrategy = CurriculumStrategy.BABY_STEP
    schedule: CompetenceSchedule = None
    initial_competence: float = 0.1
    num_epochs: int = 100
    self_paced_growth_rate: float = 1.2
    self_paced_initial_threshold: float = 0.5
    shuffle_within_subset: bool = True
    min_samples: int = 1

    def __post_init__(self):
        if self.schedule is None:
            self.schedule = CompetenceSchedule()
        if not 0 < self.initial_competence <= 1:
            raise ValueError("initial_competence must be in (0, 1]")
        if self.num_epochs <= 0 or self.min_samples <= 0:
            raise ValueError("num_epochs and min_samples must be positive")
        if self.self_paced_growth_rate <= 0 or self.self_paced_initial_threshold <= 0:
            raise ValueError("self-paced parameters must be positive")

    def competence_at(self, epoch: int) -> float:
        t = min(epoch / self.num_epochs, 1.0)
        c0 = self.initial_competence
        s = self.schedule
        if s.kind == "linear":
            c = c0 + (1 - c0) * t
        elif s.kind == "sqrt":
            c = c0 + (1 - c0) * math.sqrt(t)
        else:
            step = min(math.ceil(t * s.num_steps), s.num_steps)
            c = c0 + (1 - c0) * step / s.num_steps
        return max(min(c, 1.0), c0)


class CurriculumLearner:
    def __init__(self, config: CurriculumConfig, difficulties, seed: int = 0):
        self.config = config
        self.difficulties = [min(max(float(d), 0.0), 1.0) for d in difficulties]
        n = self.num_samples = len(self.difficulties)
        rev = config.strategy == CurriculumStrategy.ANTI_CURRICULUM
        self.sorted_indices = sorted(range(n), key=lambda i: self.difficulties[i], reverse=rev)
        self.sample_losses = [0.0] * n
        self.self_paced_threshold = config.self_paced_initial_threshold
        self.epoch_sample_counts: list[int] = []
        self._rng = random.Random(seed)

    def competence(self, epoch: int) -> float:
        return self.config.competence_at(epoch)

    def _count(self, c: float) -> int:
        return min(max(math.ceil(c * self.num_samples), self.config.min_samples), self.num_samples)

    def get_batch_indices(self, epoch: int) -> list[int]:
        s = self.config.strategy
        if s in (CurriculumStrategy.BABY_STEP, CurriculumStrategy.ANTI_CURRICULUM):
            idx = self.sorted_indices[: self._count(self.competence(epoch))]
        elif s == CurriculumStrategy.ONE_PASS:
            prev = self.competence(epoch - 1) if epoch > 0 else 0.0
            start = min(math.floor(prev * self.num_samples), self.num_samples)
            end = self._count(self.competence(epoch))
            if start >= end:
                start = max(end - self.config.min_samples, 0)
            idx = self.sorted_indices[start:end]
        else:
            idx = [i for i in range(self.num_samples) if self.sample_losses[i] < self.self_paced_threshold]
            have = set(idx)
            for i in self.sorted_indices:
                if len(idx) >= self.config.min_samples:
                    break
                if i not in have:
                    idx.append(i)
        idx = list(idx)
        if self.config.shuffle_within_subset:
            self._rng.shuffle(idx)
        self.epoch_sample_counts.append(len(idx))
        return idx

    def update_losses(self, losses):
        if len(losses) != self.num_samples:
            raise ValueError("one loss per sample")
        self.sample_losses = [float(x) for x in losses]
        self.self_paced_threshold *= self.config.self_paced_growth_rate

    def update_difficulties(self, d):
        self.__init__(self.config, d)
