"""Hyperparameter search: grid, random, successive halving and a basic
tree-structured Parzen estimator over a typed search space.

Reference parity: scirs2-neural/src/training/hparam_tuner.rs:51-1190
(HParamValue, HParamSpace uniform / log_uniform / int_range / choice /
boolean, SearchStrategy Grid / Random / SuccessiveHalving / TPE,
TrialResult, best configuration).
"""
from __future__ import annotations

import itertools
import math
import random
from dataclasses import dataclass, field


@dataclass
class HParamSpace:
    name: str
    kind: str                      # uniform | log_uniform | int | choice | bool
    low: float = 0.0
    high: float = 1.0
    values: list = field(default_factory=list)

    @staticmethod
    def uniform(name, low, high):
        return HParamSpace(name, "uniform", low, high)

    @staticmethod
    def log_uniform(name, low, high):
        if low <= 0:
            raise ValueError("log_uniform needs low > 0")
        return HParamSpace(name, "log_uniform", low, high)

    @staticmethod
    def int_range(name, low, high):
        return HParamSpace(name, "int", low, high)

    @staticmethod
    def choice(name, values):
        return HParamSpace(name, "choice", values=list(values))

    @staticmethod
    def boolean(name):
        return HParamSpace(name, "bool", values=[False, True])

    def sample(self, rng: random.Random):
        if self.kind == "uniform":
            return rng.uniform(self.low, self.high)
        if self.kind == "log_uniform":
            return math.exp(rng.uniform(math.log(self.low), math.log(self.high)))
        if self.kind == "int":
            return rng.randint(int(self.low), int(self.high))
        return rng.choice(self.values)

    def grid(self, n: int) -> list:
        if self.kind in ("choice", "bool"):
            return list(self.values)
        if self.kind == "int":
            lo, hi = int(self.low), int(self.high)
            if hi - lo + 1 <= n:
                return list(range(lo, hi + 1))
            return sorted({round(lo + (hi - lo) * i / (n - 1)) for i in range(n)})
        if n == 1:
            return [(self.low + self.high) / 2]
        if self.kind == "log_uniform":
            a, b = math.log(self.low), math.log(self.high)
            return [math.exp(a + (b - a) * i / (n - 1)) for i in range(n)]
        return [self.low + (self.high - self.low) * i / (n - 1) for i in range(n)]

    # position in [0, 1] (TPE works on these)
    def to_unit(self, v) -> float:
        if self.kind == "uniform":
            return (v - self.low) / (self.high - self.low or 1)
        if self.kind == "log_uniform":
            return (math.log(v) - math.log(self.low)) / (math.log(self.high) - math.log(self.low) or 1)
        if self.kind == "int":
            return (v - self.low) / ((self.high - self.low) or 1)
        return self.values.index(v) / max(len(self.values) - 1, 1)

    def from_unit(self, u: float):
        u = min(max(u, 0.0), 1.0)
        if self.kind == "uniform":
            return self.low + u * (self.high - self.low)
        if self.kind == "log_uniform":
            return math.exp(math.log(self.low) + u * (math.log(self.high) - math.log(self.low)))
        if self.kind == "int":
            return int(round(self.low + u * (self.high - self.low)))
        return self.values[int(round(u * (len(self.values) - 1)))]


@dataclass
class SearchStrategy:
    kind: str                          # grid | random | successive_halving | tpe
    points_per_dim: int = 3
    max_trials: int = 20
    max_resource: int = 27
    reduction_factor: int = 3
    num_initial: int = 27
    n_startup: int = 5
    gamma: float = 0.25

    @staticmethod
    def grid(points_per_dim=3):
        return SearchStrategy("grid", points_per_dim=points_per_dim)

    @staticmethod
    def random_search(max_trials=20):
        return SearchStrategy("random", max_trials=max_trials)

    @staticmethod
    def successive_halving(max_resource=27, reduction_factor=3, num_initial=27):
        return SearchStrategy("successive_halving", max_resource=max_resource, reduction_factor=reduction_factor,
                              num_initial=num_initial)

    @staticmethod
    def tpe(max_trials=30, n_startup=5, gamma=0.25):
        return SearchStrategy("tpe", max_trials=max_trials, n_startup=n_startup, gamma=gamma)


@dataclass
class TrialResult:
    trial_id: int
    config: dict
    score: float
    resource: int = 1


class HParamTuner:
    """`objective(config, resource) -> score`; lower is better unless
    `maximize` is set."""

    def __init__(self, spaces: list[HParamSpace], strategy: SearchStrategy, maximize: bool = False, seed: int = 0):
        self.spaces, self.strategy, self.maximize = spaces, strategy, maximize
        self.rng = random.Random(seed)
        self.trials: list[TrialResult] = []

    def _better(self, a: float, b: float) -> bool:
        return a > b if self.maximize else a < b

    def _sample(self) -> dict:
        return {s.name: s.sample(self.rng) for s in self.spaces}

    def _eval(self, objective, config, resource=1) -> TrialResult:
        r = TrialResult(len(self.trials), dict(config), float(objective(config, resource)), resource)
        self.trials.append(r)
        return r

    def run(self, objective) -> TrialResult:
        st = self.strategy
        if st.kind == "grid":
            names = [s.name for s in self.spaces]
            for combo in itertools.product(*[s.grid(st.points_per_dim) for s in self.spaces]):
                self._eval(objective, dict(zip(names, combo)))
        elif st.kind == "random":
            for _ in range(st.max_trials):
                self._eval(objective, self._sample())
        elif st.kind == "successive_halving":
            configs = [self._sample() for _ in range(st.num_initial)]
            resource = max(1, st.max_resource // st.reduction_factor ** max(
                0, int(math.log(max(st.num_initial, 1), st.reduction_factor))))
            while configs:
                res = [self._eval(objective, c, resource) for c in configs]
                if len(configs) == 1 or resource >= st.max_resource:
                    break
                res.sort(key=lambda t: -t.score if self.maximize else t.score)
                configs = [t.config for t in res[:max(1, len(res) // st.reduction_factor)]]
                resource = min(st.max_resource, resource * st.reduction_factor)
        elif st.kind == "tpe":
            for i in range(st.max_trials):
                self._eval(objective, self._sample() if i < st.n_startup else self._tpe_suggest())
        else:
            raise ValueError(st.kind)
        return self.best()

    def _tpe_suggest(self, candidates: int = 24) -> dict:
        done = sorted(self.trials, key=lambda t: -t.score if self.maximize else t.score)
        n_good = max(1, int(math.ceil(self.strategy.gamma * len(done))))
        good, bad = done[:n_good], done[n_good:] or done[-1:]
        bw = 0.15

        def density(u, pts):
            return sum(math.exp(-0.5 * ((u - p) / bw) ** 2) for p in pts) / (len(pts) * bw) + 1e-12

        cfg = {}
        for s in self.spaces:
            gpts = [s.to_unit(t.config[s.name]) for t in good]
            bpts = [s.to_unit(t.config[s.name]) for t in bad]
            cands = [self.rng.choice(gpts) + self.rng.gauss(0, bw) for _ in range(candidates)]
            best = max(cands, key=lambda u: density(u, gpts) / density(u, bpts))
            cfg[s.name] = s.from_unit(best)
        return cfg

    def best(self) -> TrialResult:
        top = [t for t in self.trials if t.resource == max(x.resource for x in self.trials)]
        return max(top, key=lambda t: t.score) if self.maximize else min(top, key=lambda t: t.score)
