"""Parameter-efficient fine-tuning adapters.

  LoRALinear   scirs2-neural/src/lora/linear.rs:89-338   y = x W^T + (alpha/r) x A^T B^T,
               A ~ Kaiming-uniform (gain sqrt 2) [r, in], B = 0 [out, r]; merge / unmerge
  DoRALinear   scirs2-neural/src/lora/dora.rs:33-215     magnitude * row-normalised (W + s B A)
  IA3Adapter   scirs2-neural/src/lora/ia3.rs:38-201      learned per-feature scale (init 1)
  VeRALinear   scirs2-neural/src/lora/vera.rs:260-560    frozen shared random A, B; trainable
               scaling vectors d (init d_init) and b (init 0)
  AdaLoRALinear  scirs2-neural/src/lora/adalora.rs:32-260  U diag(s) V with an importance-pruned rank budget
  BottleneckAdapter  scirs2-neural/src/lora/adapter.rs:82-280  down -> activation -> up (+ residual)
  merge_lora_weights / merge_multiple_lora / quantize_merged_weight  scirs2-neural/src/lora/merge.rs

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


# ---------------------------------------------------------------------------- AdaLoRA
@dataclass
class AdaLoraConfig:
    """AdaLoRA (Zhang et al. 2023): the update is P diag(lambda) Q with a rank budget
    pruned by an importance score. Field names and defaults follow
    scirs2-neural/src/lora/adalora.rs:32-80."""

    initial_rank: int = 12
    target_rank: int = 4
    delta_t: int = 10
    beta1: float = 0.85
    beta2: float = 0.85
    alpha: float = 1.0
    seed: int = 42


class AdaLoRALinear(Layer):
    """y = x W^T + x (U diag(s * alpha / r * mask) V)^T with W frozen.

    U [out, r] and V [r, in] start as small Gaussians and s as zeros (the
    published initialisation, so every factor receives gradients; the
    reference starts U = V = 0 and s = 0.01, which also gives W_eff = W but
    leaves U and V without gradient). `update_importance` keeps an EMA of the
    sensitivity |s * ds| per rank, `prune_to_budget` keeps the most important
    `budget` ranks (the mask), `budget_at(step, total)` is a cubic schedule
    from initial_rank to target_rank after delta_t warm-up steps.
    Reference parity: scirs2-neural/src/lora/adalora.rs:85-260."""

    def __init__(self, weight: torch.Tensor, config: AdaLoraConfig | None = None, bias: torch.Tensor | None = None):
        super().__init__()
        c = config or AdaLoraConfig()
        if c.initial_rank <= 0:
            raise ValueError("AdaLoRA initial_rank must be > 0")
        if c.target_rank > c.initial_rank:
            raise ValueError(f"AdaLoRA target_rank {c.target_rank} must be <= initial_rank {c.initial_rank}")
        out_f, in_f = weight.shape
        r = c.initial_rank
        self.config = c
        self.weight = nn.Parameter(weight.detach().clone(), requires_grad=False)
        self.bias = None if bias is None else nn.Parameter(bias.detach().clone(), requires_grad=False)
        g = torch.Generator().manual_seed(c.seed)
        self.u_mat = nn.Parameter((torch.randn(out_f, r, generator=g) * 0.02).to(weight))
        self.v_mat = nn.Parameter((torch.randn(r, in_f, generator=g) * 0.02).to(weight))
        self.singular_values = nn.Parameter(torch.zeros(r, dtype=weight.dtype, device=weight.device))
        self.register_buffer("importance_ema", torch.zeros(r, dtype=torch.float32, device=weight.device))
        self.register_buffer("rank_mask", torch.ones(r, dtype=weight.dtype, device=weight.device))
        self.scaling = c.alpha / r

    def _lam(self):
        return self.singular_values * self.scaling * self.rank_mask

    def delta_weight(self):
        return (self.u_mat * self._lam()) @ self.v_mat

    def effective_weight(self):
        return self.weight + self.delta_weight()

    def forward(self, x):
        if x.shape[-1] != self.weight.shape[1]:
            raise ValueError(f"AdaLoRA expects {self.weight.shape[1]} input features, got {x.shape[-1]}")
        y = FN.linear(x, self.weight.t(), self.bias)
        h = FN.linear(x, self.v_mat.t()) * self._lam()
        return y + FN.linear(h, self.u_mat.t())

    @torch.no_grad()
    def update_importance(self, grad_s: torch.Tensor | None = None):
        """EMA of |s * dL/ds| per rank (dL/ds from `grad_s` or the parameter's .grad)."""
        g = grad_s if grad_s is not None else self.singular_values.grad
        if g is None or g.numel() != self.config.initial_rank:
            raise ValueError(f"update_importance: expected a gradient of length {self.config.initial_rank}")
        sens = (self.singular_values.float() * g.float()).abs()
        b = self.config.beta1
        self.importance_ema.mul_(b).add_((1.0 - b) * sens)

    @torch.no_grad()
    def prune_to_budget(self, budget: int) -> int:
        keep = min(int(budget), self.config.initial_rank)
        order = torch.argsort(self.importance_ema, descending=True, stable=True)
        self.rank_mask.zero_()
        self.rank_mask[order[:keep]] = 1.0
        return keep

    def budget_at(self, step: int, total_steps: int) -> int:
        c = self.config
        if step <= c.delta_t or total_steps <= c.delta_t:
            return c.initial_rank
        frac = min(1.0, (step - c.delta_t) / max(1, total_steps - c.delta_t))
        return int(round(c.target_rank + (c.initial_rank - c.target_rank) * (1.0 - frac) ** 3))

    def active_rank(self) -> int:
        return int((self.rank_mask > 0.5).sum())

    def target_rank(self) -> int:
        return self.config.target_rank

    def orthogonality_penalty(self):
        """||U^T U - I||_F^2 + ||V V^T - I||_F^2 (the AdaLoRA regulariser)."""
        r = self.config.initial_rank
        eye = torch.eye(r, dtype=self.u_mat.dtype, device=self.u_mat.device)
        return ((self.u_mat.t() @ self.u_mat - eye) ** 2).sum() + ((self.v_mat @ self.v_mat.t() - eye) ** 2).sum()


# ---------------------------------------------------------------------------- bottleneck adapter
_ADAPTER_ACTS = ("relu", "gelu", "silu", "tanh")


@dataclass
class AdapterConfig:
    """Field names and defaults follow scirs2-neural/src/lora/types.rs:186-215."""

    bottleneck_dim: int = 64
    activation: str = "relu"
    residual: bool = True
    seed: int = 42

    def validate(self):
        if self.bottleneck_dim <= 0:
            raise ValueError("Adapter bottleneck_dim must be > 0")
        if self.activation.lower() not in _ADAPTER_ACTS:
            raise ValueError(f"adapter activation must be one of {_ADAPTER_ACTS}")


def _xorshift_uniform(n: int, bound: float, seed: int) -> torch.Tensor:
    """Marsaglia xorshift64 (13, 7, 17) uniforms in (-bound, bound): the generator the reference
    seeds adapters with, so equal seeds give equal initial weights."""
    state = seed if seed != 0 else 0xDEADBEEFCAFE1234
    mask = (1 << 64) - 1
    out = []
    for _ in range(n):
        state ^= (state << 13) & mask
        state ^= state >> 7
        state ^= (state << 17) & mask
        out.append(((state >> 11) / float(1 << 53) * 2.0 - 1.0) * bound)
    return torch.tensor(out, dtype=torch.float64)


class BottleneckAdapter(Layer):
    """y = x + up(act(down(x) + b_down)) + b_up (residual optional); down [bottleneck, in] and
    up [in, bottleneck] Xavier-uniform from the seeded xorshift generator, biases zero.
    Reference parity: scirs2-neural/src/lora/adapter.rs:82-280."""

    def __init__(self, input_dim: int, config: AdapterConfig | None = None, dtype=torch.float32, device=None):
        super().__init__()
        c = config or AdapterConfig()
        c.validate()
        if input_dim <= 0:
            raise ValueError("Adapter input_dim must be > 0")
        bd = c.bottleneck_dim
        # one generator stream: the down projection's values first, then the up projection's
        vals = _xorshift_uniform(bd * input_dim * 2, 1.0, c.seed)
        b1 = math.sqrt(6.0 / (input_dim + bd))
        self.down_project = nn.Parameter((vals[:bd * input_dim] * b1).view(bd, input_dim).to(dtype=dtype,
                                                                                             device=device))
        self.up_project = nn.Parameter((vals[bd * input_dim:] * b1).view(input_dim, bd).to(dtype=dtype, device=device))
        self.bias_down = nn.Parameter(torch.zeros(bd, dtype=dtype, device=device))
        self.bias_up = nn.Parameter(torch.zeros(input_dim, dtype=dtype, device=device))
        self.activation, self.residual = c.activation.lower(), c.residual
        self.input_dim, self.bottleneck_dim = input_dim, bd

    def _act(self, h):
        if self.activation == "relu":
            return torch.relu(h)
        if self.activation == "gelu":
            return 0.5 * h * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (h + 0.044715 * h ** 3)))
        if self.activation == "silu":
            return h * torch.sigmoid(h)
        return torch.tanh(h)

    def forward(self, x):
        if x.shape[-1] != self.input_dim:
            raise ValueError(f"Input has {x.shape[-1]} features but adapter expects {self.input_dim}")
        h = self._act(FN.linear(x, self.down_project.t(), self.bias_down))
        y = FN.linear(h, self.up_project.t(), self.bias_up)
        return x + y if self.residual else y

    def stats(self) -> dict:
        trainable = 2 * self.bottleneck_dim * self.input_dim + self.bottleneck_dim + self.input_dim
        return {"trainable_params": trainable, "total_params": trainable, "frozen_params": 0,
                "compression_ratio": 1.0}


# ---------------------------------------------------------------------------- merging
def merge_lora_weights(weight: torch.Tensor, a: torch.Tensor, b: torch.Tensor, scaling: float) -> torch.Tensor:
    """W + scaling * B A (W [out, in], A [r, in], B [out, r]).
    Reference parity: scirs2-neural/src/lora/merge.rs:25-60."""
    out_f, in_f = weight.shape
    if a.shape[1] != in_f:
        raise ValueError(f"A columns ({a.shape[1]}) must match weight columns ({in_f})")
    if b.shape[0] != out_f:
        raise ValueError(f"B rows ({b.shape[0]}) must match weight rows ({out_f})")
    if b.shape[1] != a.shape[0]:
        raise ValueError(f"B columns ({b.shape[1]}) must match A rows ({a.shape[0]})")
    return weight + scaling * (b @ a)


def merge_multiple_lora(base_weight: torch.Tensor, lora_params: list) -> torch.Tensor:
    """Apply merge_lora_weights for every (A, B, scaling) in order."""
    w = base_weight
    for a, b, s in lora_params:
        w = merge_lora_weights(w, a, b, s)
    return w


def compute_effective_weight(layer) -> torch.Tensor:
    """W + delta of a LoRA / DoRA / AdaLoRA layer, whether or not it is merged."""
    if isinstance(layer, AdaLoRALinear):
        return layer.effective_weight().detach()
    if isinstance(layer, LoRALinear):
        return (layer.weight if layer.merged else layer.weight + layer.lora_delta()).detach()
    if hasattr(layer, "effective_weight"):
        return layer.effective_weight().detach()
    raise TypeError(f"no effective weight for {type(layer).__name__}")


@dataclass
class QuantizedWeight:
    """Symmetric int8 weight: value = data * scale (zero point 0).
    Reference parity: scirs2-neural/src/lora/merge.rs:72-190."""

    data: torch.Tensor  # int8 [rows, cols]
    scale: float
    zero_point: int = 0
    bits: int = 8

    @property
    def rows(self):
        return self.data.shape[0]

    @property
    def cols(self):
        return self.data.shape[1]

    def dequantize(self) -> torch.Tensor:
        return (self.data.to(torch.float64) - self.zero_point) * self.scale

    def compression_ratio(self) -> float:
        return 64.0 / self.bits  # against float64 storage, as in the reference

    def quantization_error(self, original: torch.Tensor) -> float:
        """Mean absolute error of the dequantized weight."""
        if tuple(original.shape) != tuple(self.data.shape):
            raise ValueError("shape mismatch")
        return float((self.dequantize() - original.to(torch.float64)).abs().mean())


def quantize_merged_weight(weight: torch.Tensor, bits: int = 8) -> QuantizedWeight:
    if bits != 8:
        raise ValueError(f"Only 8-bit quantization is currently supported, got {bits}")
    if weight.numel() == 0:
        raise ValueError("Cannot quantize empty weight matrix")
    w = weight.detach().to(torch.float64)
    m = float(w.abs().max())
    if m < torch.finfo(torch.float64).eps:
        return QuantizedWeight(torch.zeros(w.shape, dtype=torch.int8), 1.0)
    scale = m / 127.0
    return QuantizedWeight(torch.round(w / scale).clamp(-128, 127).to(torch.int8), scale)
