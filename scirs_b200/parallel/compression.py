"""Gradient compression for bandwidth-limited synchronisation.

* Top-k with error feedback (the residual of what was not sent is added to
  the next gradient), random-k, 1-bit sign quantisation with a scale, and
  PowerSGD rank-r low-rank compression (one power iteration with a reused Q,
  orthonormalised P).
* `compressed_allreduce` applies top-k + error feedback across the process
  group (all-gather of (index, value) pairs, scatter-add, average).

All operate on torch tensors on any device. Reference parity:
scirs2-core/src/distributed/compression.rs:16-410 (TopKCompressor,
RandomKCompressor, OneBitQuantizer, PowerSgdConfig / low_rank_compress) and
scirs2-neural/src/training/gradient_compression.rs.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class TopKConfig:
    k_fraction: float = 0.01
    error_feedback: bool = True


class TopKCompressor:
    def __init__(self, n_params: int, config: TopKConfig | None = None, device=None):
        self.config = config or TopKConfig()
        self.residual = torch.zeros(n_params, device=device)

    def compress(self, grad: torch.Tensor):
        g = grad.reshape(-1).float()
        if self.config.error_feedback:
            g = g + self.residual.to(g.device)
        k = max(1, int(round(g.numel() * self.config.k_fraction)))
        idx = g.abs().topk(k).indices
        vals = g[idx]
        if self.config.error_feedback:
            self.residual = g.clone()
            self.residual[idx] = 0.0
        return idx, vals

    @staticmethod
    def decompress(idx, vals, n_total: int) -> torch.Tensor:
        out = torch.zeros(n_total, dtype=vals.dtype, device=vals.device)
        out.index_add_(0, idx, vals)
        return out

    def compression_ratio(self, n_total: int) -> float:
        k = max(1, int(round(n_total * self.config.k_fraction)))
        return n_total * 4 / (k * 12)


class RandomKCompressor:
    def __init__(self, k_fraction: float = 0.01):
        self.k_fraction = k_fraction

    def compress(self, grad: torch.Tensor, seed: int):
        g = grad.reshape(-1)
        k = max(1, int(round(g.numel() * self.k_fraction)))
        gen = torch.Generator(device="cpu").manual_seed(seed)
        idx = torch.randperm(g.numel(), generator=gen)[:k].to(g.device)
        return idx, g[idx] * (g.numel() / k)  # unbiased

    decompress = staticmethod(TopKCompressor.decompress)


class OneBitQuantizer:
    @staticmethod
    def quantize(grad: torch.Tensor):
        g = grad.reshape(-1).float()
        scale = float(g.abs().mean())
        bits = (g >= 0).to(torch.uint8)
        return bits, scale

    @staticmethod
    def dequantize(bits: torch.Tensor, scale: float, n: int) -> torch.Tensor:
        return (bits[:n].float() * 2 - 1) * scale

    @staticmethod
    def quantization_error(original: torch.Tensor, quantized: torch.Tensor) -> float:
        return float((original.reshape(-1) - quantized.reshape(-1)).norm() / original.norm().clamp(min=1e-30))


@dataclass
class PowerSgdConfig:
    rank: int = 4
    seed: int = 0


def low_rank_compress(m: torch.Tensor, rank: int = 4, q: torch.Tensor | None = None, seed: int = 0):
    """M [n, k] ~ P Q^T with P [n, r] orthonormal, Q [k, r] (one power step)."""
    m = m.float()
    if q is None:
        gen = torch.Generator(device="cpu").manual_seed(seed)
        q = torch.randn(m.shape[1], rank, generator=gen).to(m.device)
    p, _ = torch.linalg.qr(m @ q)
    q = m.t() @ p
    return p, q


def low_rank_decompress(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    return p @ q.t()


def compressed_allreduce(grad: torch.Tensor, compressor: TopKCompressor, group=None) -> torch.Tensor:
    """Average `grad` over the group sending only each rank's top-k entries."""
    idx, vals = compressor.compress(grad)
    world = dist.get_world_size(group)
    k = torch.tensor([idx.numel()], device=grad.device)
    ks = [torch.zeros_like(k) for _ in range(world)]
    dist.all_gather(ks, k, group=group)
    kmax = int(max(int(x) for x in ks))
    pi = torch.zeros(kmax, dtype=torch.long, device=grad.device)
    pv = torch.zeros(kmax, dtype=vals.dtype, device=grad.device)
    pi[: idx.numel()], pv[: vals.numel()] = idx, vals
    ai = [torch.zeros_like(pi) for _ in range(world)]
    av = [torch.zeros_like(pv) for _ in range(world)]
    dist.all_gather(ai, pi, group=group)
    dist.all_gather(av, pv, group=group)
    out = torch.zeros(grad.numel(), dtype=vals.dtype, device=grad.device)
    for kk, ii, vv in zip(ks, ai, av):
        n = int(kk)
        out.index_add_(0, ii[:n], vv[:n])
    return (out / world).view_as(grad)
