"""Federated averaging (server side) with client selection, robust
aggregation, differential privacy and update compression.

The server holds the global parameters (a list of tensors); each round it
selects clients, receives their updated parameters (ClientUpdate), clips and
noises them when differential privacy is on, optionally sparsifies the
deltas (top-k), and aggregates (FedAvg weighted by sample count, plain mean
or coordinate-wise median).

Reference parity: scirs2-neural/src/training/federated.rs:55-1272
(ClientSelectionStrategy, AggregationMethod, DifferentialPrivacyConfig,
GradientCompressionConfig, FederatedConfig + builder, ClientUpdate,
RoundStats, FederatedServer); an in-process simulation there as here.
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field

import torch


class ClientSelectionStrategy(enum.Enum):
    RANDOM = "Random"
    IMPORTANCE_BASED = "ImportanceBased"
    ALL = "All"


class AggregationMethod(enum.Enum):
    FED_AVG = "FedAvg"
    SIMPLE_MEAN = "SimpleMean"
    MEDIAN = "Median"


@dataclass
class DifferentialPrivacyConfig:
    noise_multiplier: float = 1.0
    max_grad_norm: float = 1.0
    delta: float = 1e-5


@dataclass
class GradientCompressionConfig:
    top_k_fraction: float = 0.1


@dataclass
class FederatedConfig:
    num_rounds: int = 10
    clients_per_round: int = 10
    client_selection: ClientSelectionStrategy = ClientSelectionStrategy.RANDOM
    aggregation: AggregationMethod = AggregationMethod.FED_AVG
    differential_privacy: DifferentialPrivacyConfig | None = None
    gradient_compression: GradientCompressionConfig | None = None
    local_epochs: int = 1
    local_lr: float = 0.01
    seed: int = 0

    @staticmethod
    def builder() -> "FederatedConfigBuilder":
        return FederatedConfigBuilder()

    def validate(self):
        if self.num_rounds <= 0 or self.clients_per_round <= 0 or self.local_epochs <= 0:
            raise ValueError("rounds, clients per round and local epochs must be positive")
        if self.local_lr <= 0:
            raise ValueError("local learning rate must be positive")
        dp = self.differential_privacy
        if dp is not None and (dp.noise_multiplier < 0 or dp.max_grad_norm <= 0 or not 0 < dp.delta < 1):
            raise ValueError("invalid differential privacy settings")
        gc = self.gradient_compression
        if gc is not None and not 0 < gc.top_k_fraction <= 1:
            raise ValueError("top_k_fraction must be in (0, 1]")


class FederatedConfigBuilder:
    def __init__(self):
        self.c = FederatedConfig()

    def num_rounds(self, n):
        self.c.num_rounds = n
        return self

    def clients_per_round(self, n):
        self.c.clients_per_round = n
        return self

    def client_selection(self, s):
        self.c.client_selection = s
        return self

    def aggregation(self, a):
        self.c.aggregation = a
        return self

    def differential_privacy(self, noise_multiplier, max_grad_norm):
        self.c.differential_privacy = DifferentialPrivacyConfig(noise_multiplier, max_grad_norm)
        return self

    def dp_delta(self, delta):
        if self.c.differential_privacy is None:
            self.c.differential_privacy = DifferentialPrivacyConfig()
        self.c.differential_privacy.delta = delta
        return self

    def gradient_compression(self, top_k_fraction):
        self.c.gradient_compression = GradientCompressionConfig(top_k_fraction)
        return self

    def local_epochs(self, n):
        self.c.local_epochs = n
        return self

    def local_lr(self, lr):
        self.c.local_lr = lr
        return self

    def seed(self, s):
        self.c.seed = s
        return self

    def build(self) -> FederatedConfig:
        self.c.validate()
        return self.c


@dataclass
class ClientUpdate:
    client_id: int
    parameters: list
    num_samples: int
    loss: float | None = None
    metrics: dict = field(default_factory=dict)

    def with_loss(self, loss):
        self.loss = loss
        return self

    def with_metric(self, name, value):
        self.metrics[name] = value
        return self


@dataclass
class RoundStats:
    round: int
    num_clients: int
    mean_loss: float | None
    update_norm: float
    epsilon: float | None = None


class FederatedServer:
    def __init__(self, config: FederatedConfig, global_params: list):
        config.validate()
        self.config = config
        self.params = [p.detach().clone().float() for p in global_params]
        self.round = 0
        self.history: list[RoundStats] = []
        self.gen = torch.Generator().manual_seed(config.seed)
        self.importance: dict[int, float] = {}

    def global_params(self):
        return self.params

    def current_round(self) -> int:
        return self.round

    def round_history(self):
        return self.history

    def is_complete(self) -> bool:
        return self.round >= self.config.num_rounds

    def select_clients(self, num_clients: int) -> list[int]:
        c = self.config
        k = min(c.clients_per_round, num_clients)
        if c.client_selection == ClientSelectionStrategy.ALL:
            return list(range(num_clients))
        if c.client_selection == ClientSelectionStrategy.IMPORTANCE_BASED and self.importance:
            w = torch.tensor([self.importance.get(i, 1.0) for i in range(num_clients)], dtype=torch.float64)
            return sorted(torch.multinomial(w, k, replacement=False, generator=self.gen).tolist())
        return sorted(torch.randperm(num_clients, generator=self.gen)[:k].tolist())

    def _privatise(self, delta: list) -> list:
        dp = self.config.differential_privacy
        norm = math.sqrt(sum(float((d ** 2).sum()) for d in delta))
        s = min(1.0, dp.max_grad_norm / max(norm, 1e-12))
        return [d * s for d in delta]

    def _compress(self, delta: list) -> list:
        out = []
        for d in delta:
            f = d.reshape(-1)
            k = max(1, int(round(f.numel() * self.config.gradient_compression.top_k_fraction)))
            keep = torch.zeros_like(f)
            idx = f.abs().topk(k).indices
            keep[idx] = f[idx]
            out.append(keep.view_as(d))
        return out

    def aggregate(self, updates: list[ClientUpdate]) -> RoundStats:
        c = self.config
        deltas = [[p.float() - g for p, g in zip(u.parameters, self.params)] for u in updates]
        if c.differential_privacy is not None:
            deltas = [self._privatise(d) for d in deltas]
        if c.gradient_compression is not None:
            deltas = [self._compress(d) for d in deltas]
        agg = []
        for j in range(len(self.params)):
            stack = torch.stack([d[j] for d in deltas])
            if c.aggregation == AggregationMethod.FED_AVG:
                w = torch.tensor([u.num_samples for u in updates], dtype=stack.dtype)
                w = (w / w.sum()).view(-1, *([1] * (stack.dim() - 1)))
                a = (stack * w).sum(0)
            elif c.aggregation == AggregationMethod.SIMPLE_MEAN:
                a = stack.mean(0)
            else:
                a = stack.median(0).values
            agg.append(a)
        eps = None
        if c.differential_privacy is not None:
            dp = c.differential_privacy
            sigma = dp.noise_multiplier * dp.max_grad_norm / len(updates)
            agg = [a + torch.randn(a.shape, generator=self.gen) * sigma for a in agg]
            q = len(updates) / max(len(updates), c.clients_per_round)
            # Gaussian-mechanism composition bound over the rounds so far
            eps = q * math.sqrt(2 * (self.round + 1) * math.log(1 / dp.delta)) / max(dp.noise_multiplier, 1e-12)
        self.params = [g + a for g, a in zip(self.params, agg)]
        for u, d in zip(updates, deltas):
            self.importance[u.client_id] = 1.0 + math.sqrt(sum(float((x ** 2).sum()) for x in d))
        losses = [u.loss for u in updates if u.loss is not None]
        st = RoundStats(self.round, len(updates), sum(losses) / len(losses) if losses else None,
                        math.sqrt(sum(float((a ** 2).sum()) for a in agg)), eps)
        self.history.append(st)
        self.round += 1
        return st
