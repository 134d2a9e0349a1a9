"""Speculative decoding by rejection sampling (Leviathan et al., 2023).

A cheap draft model proposes `draft_steps` tokens; the target model scores
them in one pass; each draft token x is kept with probability
min(1, p_target(x) / p_draft(x)) (optionally floored by
`acceptance_threshold`), and at the first rejection a correction token is
drawn from the residual max(0, p_target - p_draft) renormalised. When all
are kept, a bonus token is drawn from the last target distribution. With a
zero floor the output distribution equals the target model's.

Distributions are torch tensors (any device); sampling uses a Marsaglia
xorshift64 generator so runs are reproducible from a seed.

Reference parity: scirs2-neural/src/inference/speculative/types.rs:23-143
(SpeculativeConfig, SpeculativeResult) and rejection_sampling.rs:46-667
(Xorshift64, TokenDist, SpeculativeDecoder::rejection_sampling_step / decode).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class SpeculativeConfig:
    draft_steps: int = 4
    temperature: float = 1.0
    top_p: float = 0.9
    max_tokens: int = 256
    acceptance_threshold: float = 0.0


@dataclass
class SpeculativeResult:
    accepted_tokens: list = field(default_factory=list)
    n_draft_tokens: int = 0
    n_accepted_tokens: int = 0
    n_steps: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.n_accepted_tokens / self.n_draft_tokens if self.n_draft_tokens else 0.0


class Xorshift64:
    """Marsaglia's 64-bit xorshift generator (shifts 13, 7, 17)."""

    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        self.state = (seed & self.MASK) or 0x9E3779B97F4A7C15

    def next_u64(self) -> int:
        x = self.state
        x ^= (x << 13) & self.MASK
        x ^= x >> 7
        x ^= (x << 17) & self.MASK
        self.state = x
        return x

    def next_f64(self) -> float:
        return (self.next_u64() >> 11) / float(1 << 53)


def _probs(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    t = max(float(temperature), 1e-6)
    return torch.softmax(logits.double() / t, dim=-1)


def _top_p(p: torch.Tensor, top_p: float) -> torch.Tensor:
    if top_p >= 1.0:
        return p
    srt, idx = torch.sort(p, descending=True)
    keep = torch.cumsum(srt, 0) - srt < top_p  # smallest prefix reaching top_p
    keep[0] = True
    out = torch.zeros_like(p)
    out[idx[keep]] = srt[keep]
    return out / out.sum()


def _sample(p: torch.Tensor, u: float) -> int:
    c = torch.cumsum(p, 0)
    i = int(torch.searchsorted(c, torch.tensor([u * float(c[-1])], dtype=c.dtype, device=c.device)))
    return min(i, p.numel() - 1)


class TokenDist:
    def __init__(self, logits):
        self.logits = torch.as_tensor(logits, dtype=torch.float64)

    def softmax(self) -> torch.Tensor:
        return _probs(self.logits, 1.0)

    def sample(self, temperature: float, rng: Xorshift64) -> int:
        return _sample(_probs(self.logits, temperature), rng.next_f64())

    def sample_top_p(self, temperature: float, top_p: float, rng: Xorshift64) -> int:
        return _sample(_top_p(_probs(self.logits, temperature), top_p), rng.next_f64())

    def prob(self, token: int, temperature: float) -> float:
        p = _probs(self.logits, temperature)
        return float(p[token]) if 0 <= token < p.numel() else 0.0


class SpeculativeDecoder:
    @staticmethod
    def accept_or_reject(q: float, p: float, threshold: float, rng: Xorshift64) -> bool:
        if q <= 0.0:
            return p > 0.0
        ratio = max(min(1.0, p / q), threshold)
        return rng.next_f64() < ratio

    @staticmethod
    def rejection_sampling_step(draft_logits, target_logits, draft_tokens, config: SpeculativeConfig,
                                rng: Xorshift64 | None = None):
        """Returns (accepted prefix, correction-or-bonus token)."""
        n = min(len(draft_tokens), len(draft_logits), len(target_logits))
        if n == 0:
            return [], 0
        if rng is None:
            rng = Xorshift64(int(draft_tokens[0]) * 0x9E3779B97F4A7C15 + len(draft_logits[0]))
        out = []
        for i in range(n):
            x = int(draft_tokens[i])
            qd = _top_p(_probs(torch.as_tensor(draft_logits[i]), config.temperature), config.top_p)
            pt = _top_p(_probs(torch.as_tensor(target_logits[i]), config.temperature), config.top_p)
            if SpeculativeDecoder.accept_or_reject(float(qd[x]), float(pt[x]), config.acceptance_threshold, rng):
                out.append(x)
                continue
            resid = torch.clamp(pt - qd, min=0.0)
            if float(resid.sum()) <= 0.0:
                resid = pt
            return out, _sample(resid / resid.sum(), rng.next_f64())
        last = _top_p(_probs(torch.as_tensor(target_logits[n - 1]), config.temperature), config.top_p)
        return out, _sample(last, rng.next_f64())

    @staticmethod
    def decode(context, draft_fn, target_fn, config: SpeculativeConfig, seed: int = 1) -> SpeculativeResult:
        """draft_fn(ctx) -> [(token, logits)] (up to draft_steps);
        target_fn(ctx, draft_tokens) -> [logits] (one per draft position)."""
        rng = Xorshift64(seed)
        ctx = list(context)
        res = SpeculativeResult()
        while len(res.accepted_tokens) < config.max_tokens:
            drafts = draft_fn(ctx)[: config.draft_steps]
            if not drafts:
                break
            toks = [int(t) for t, _ in drafts]
            tl = target_fn(ctx, toks)
            acc, extra = SpeculativeDecoder.rejection_sampling_step([lg for _, lg in drafts], tl, toks, config, rng)
            res.n_steps += 1
            res.n_draft_tokens += len(toks)
            res.n_accepted_tokens += len(acc)
            new = acc + [extra]
            room = config.max_tokens - len(res.accepted_tokens)
            new = new[:room]
            res.accepted_tokens += new
            ctx += new
        return res
