"""Parameter-efficient fine-tuning adapters.

  LoRALinear   scirs2-neural/src/lora/linear.rs:89-338   y = x W^T + (alpha/r) x A^T B^T,
               A ~ Kaiming-uniform (gain sqrt 2) [r, in], B = 0 [out, r]; merge / unmerge
  DoRALinear   scirs2-neural/src/lora/dora.rs:33-215     magnitude * row-normalised (W + s B A)
  IA3Adapter   scirs2-neural/src/lora/ia3.rs:38-201      learned per-feature scale (init 1)
  VeRALinear   scirs2-neural/src/lora/vera.rs:260-560    frozen shared random A, B; trainable
               scaling vectors d (init d_init) and b (init 0)

The base weight uses the torch/PyTorch layout [out, in] as in the reference
adapters. On bf16 CUDA tensors the base and low-rank products run on the
framework's tensor-core GEMM.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from ..ops import functional as FN
from .base import Layer


@dataclass
class LoRAConfig:
    rank: int = 8
    alpha: float = 16.0
    dropout: float = 0.0
    targets: list = field(default_factory=lambda: ["query", "value"])
    seed: int = 42

    def scaling(self) -> float:
        return 0.0 if self.rank == 0 else self.alpha / self.rank


def _kaiming_bound(fan_in: int) -> float:
    return math.sqrt(2.0) / math.sqrt(fan_in) * math.sqrt(3.0)


class LoRALinear(Layer):
    def __init__(self, weight: torch.Tensor, config: LoRAConfig | None = None, bias: torch.Tensor | None = None):
        super().__init__()
        config = config or LoRAConfig()
        out_f, in_f = weight.shape
        if config.rank > min(in_f, out_f):
            raise ValueError(f"LoRA rank {config.rank} exceeds min(in={in_f}, out={out_f})")
        self.weight = nn.Parameter(weight.detach().clone(), requires_grad=False)
        self.bias = None if bias is None else nn.Parameter(bias.detach().clone(), requires_grad=False)
        g = torch.Generator().manual_seed(config.seed)
        b = _kaiming_bound(in_f)
        self.lora_a = nn.Parameter(((torch.rand(config.rank, in_f, generator=g) * 2 - 1) * b).to(weight))
        self.lora_b = nn.Parameter(torch.zeros(out_f, config.rank, dtype=weight.dtype, device=weight.device))
        self._rank, self._alpha, self._scaling = config.rank, config.alpha, config.scaling()
        self.dropout = config.dropout
        self.merged = False

    def forward(self, x):
        y = FN.linear(x, self.weight.t(), self.bias)
        if self.merged or self._rank == 0:
            return y
        h = x if self.dropout == 0 or not self.training else torch.nn.functional.dropout(x, self.dropout)
        return y + (h @ self.lora_a.t() @ self.lora_b.t()) * self._scaling

    def lora_delta(self) -> torch.Tensor:
        return (self.lora_b @ self.lora_a) * self._scaling

    def effective_weight(self) -> torch.Tensor:
        return self.weight if self.merged else self.weight + self.lora_delta()

    @torch.no_grad()
    def merge(self):
        if not self.merged:
            self.weight.add_(self.lora_delta())
            self.merged = True

    @torch.no_grad()
    def unmerge(self):
        if self.merged:
            self.weight.sub_(self.lora_delta())
            self.merged = False

    def rank(self):
        return self._rank

    def alpha(self):
        return self._alpha

    def scaling(self):
        return self._scaling

    def is_merged(self):
        return self.merged

    def effective_rank(self, threshold: float = 1e-6) -> int:
        s = torch.linalg.svdvals(self.lora_delta().float())
        return int((s > threshold).sum())

    def stats(self) -> dict:
        base = self.weight.numel()
        lora = self.lora_a.numel() + self.lora_b.numel()
        return {"base_params": base, "lora_params": lora, "compression_ratio": base / max(lora, 1)}


@dataclass
class DoraConfig:
    rank: int = 8
    alpha: float = 16.0
    column_norm_eps: float = 1e-8


class DoRALinear(Layer):
    def __init__(self, weight: torch.Tensor, config: DoraConfig | None = None):
        super().__init__()
        config = config or DoraConfig()
        out_f, in_f = weight.shape
        if config.rank == 0 or config.rank > min(in_f, out_f):
            raise ValueError("invalid DoRA rank")
        self.config = config
        self.weight = nn.Parameter(weight.detach().clone(), requires_grad=False)
        self.lora_a = nn.Parameter(torch.full((config.rank, in_f), 0.02, dtype=weight.dtype, device=weight.device))
        self.lora_b = nn.Parameter(torch.zeros(out_f, config.rank, dtype=weight.dtype, device=weight.device))
        self.magnitude = nn.Parameter(weight.detach().norm(dim=1).clamp(min=config.column_norm_eps))
        self.scaling = config.alpha / config.rank

    def effective_weight(self):
        adapted = self.weight + (self.lora_b @ self.lora_a) * self.scaling
        norms = adapted.norm(dim=1, keepdim=True).clamp(min=self.config.column_norm_eps)
        return adapted * (self.magnitude[:, None] / norms)

    def forward(self, x):
        return x @ self.effective_weight().t()

    @torch.no_grad()
    def merge_into_base(self):
        self.weight.copy_(self.effective_weight())
        self.lora_b.zero_()
        self.magnitude.copy_(self.weight.norm(dim=1).clamp(min=self.config.column_norm_eps))

    def n_trainable_params(self):
        return self.lora_a.numel() + self.lora_b.numel() + self.magnitude.numel()


@dataclass
class Ia3Config:
    scale_keys: bool = True
    scale_values: bool = True
    scale_ffn: bool = True


class IA3Adapter(Layer):
    def __init__(self, dim: int, config: Ia3Config | None = None, dtype=torch.float32, device=None):
        super().__init__()
        self.config = config or Ia3Config()
        self.scale = nn.Parameter(torch.ones(dim, dtype=dtype, device=device))

    def forward(self, x):
        return x * self.scale

    def merge_into_weight_rows(self, w):
        return w * self.scale[:, None]

    def merge_into_weight_cols(self, w):
        return w * self.scale[None, :]

    def n_params(self):
        return self.scale.numel()


@dataclass
class VeRAConfig:
    rank: int = 256
    d_init: float = 0.1
    seed: int = 42


class VeRALinear(Layer):
    """W + diag(b) B diag(d) A with frozen random A [r, in], B [out, r]."""

    def __init__(self, weight: torch.Tensor, config: VeRAConfig | None = None):
        super().__init__()
        config = config or VeRAConfig()
        out_f, in_f = weight.shape
        r = config.rank
        g = torch.Generator().manual_seed(config.seed)
        self.weight = nn.Parameter(weight.detach().clone(), requires_grad=False)
        self.register_buffer("A", ((torch.rand(r, in_f, generator=g) * 2 - 1) * _kaiming_bound(in_f)).to(weight))
        self.register_buffer("B", ((torch.rand(out_f, r, generator=g) * 2 - 1) * _kaiming_bound(r)).to(weight))
        self.d = nn.Parameter(torch.full((r,), config.d_init, dtype=weight.dtype, device=weight.device))
        self.b = nn.Parameter(torch.zeros(out_f, dtype=weight.dtype, device=weight.device))
        self.merged = False

    def delta_weight(self):
        return self.b[:, None] * (self.B @ (self.d[:, None] * self.A))

    def effective_weight(self):
        return self.weight if self.merged else self.weight + self.delta_weight()

    def forward(self, x):
        return x @ self.effective_weight().t()

    @torch.no_grad()
    def merge(self):
        if not self.merged:
            self.weight.add_(self.delta_weight())
            self.merged = True

    @torch.no_grad()
    def unmerge(self):
        if self.merged:
            self.weight.sub_(self.delta_weight())
            self.merged = False

    def n_trainable_params(self):
        return self.d.numel() + self.b.numel()


def apply_lora(module: nn.Module, config: LoRAConfig, target_names=("query", "value", "w_query", "w_value")):
    """Freeze `module` and wrap every nn.Linear whose attribute name contains a
    target name in a LoRALinear. Returns the number of wrapped layers."""
    n = 0
    for p in module.parameters():
        p.requires_grad_(False)
    for name, child in list(module.named_children()):
        if isinstance(child, nn.Linear) and any(t in name for t in target_names):
            setattr(module, name, LoRALinear(child.weight, config, child.bias))
            n += 1
        else:
            n += apply_lora(child, config, target_names)
    return n
