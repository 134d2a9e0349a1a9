"""Post-training weight quantization methods and calibration.

* GPTQ (Frantar et al., 2022): columns are quantized one at a time in the
  order of the input features; each column's rounding error is spread over
  the not-yet-quantized columns with the inverse Hessian H = 2 X^T X / n of
  the layer inputs (Cholesky factor of H^-1, dampened), block by block.
* AWQ (Lin et al., 2023): input channels with large activations are scaled
  up before group quantization (s = a^alpha, alpha grid-searched to minimise
  the output error on calibration inputs) and the scale is folded back.
* SmoothQuant (Xiao et al., 2022): migrates activation outliers into the
  weights with s_j = max|X_j|^alpha / max|W_j|^(1 - alpha).
* Observers (min/max, percentile, moving average) and a calibration runner;
  post-training quantizer; quantization-aware training with fake quantization
  (straight-through estimator).

All run as PyTorch tensor code on the tensors' device (GPU or CPU).
Reference parity: scirs2-neural/src/quantization/gptq.rs:16-300,
awq.rs:42-520, smoothquant.rs, calibration.rs:17-365, qat.rs, mod.rs:230-420.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from .core import QuantizationConfig, QuantizationParams, QuantizationScheme, fake_quantize


def _group_quant(w: torch.Tensor, bits: int, group_size: int, symmetric: bool):
    """Quantize-dequantize w [out, in] per (row, group of input columns);
    returns (w_hat, scales, zeros)."""
    out_f, in_f = w.shape
    gs = in_f if group_size <= 0 else group_size
    pad = (-in_f) % gs
    x = torch.cat([w, w.new_zeros(out_f, pad)], dim=1).view(out_f, -1, gs)
    if symmetric:
        qmax = (1 << (bits - 1)) - 1
        scale = (x.abs().amax(dim=2) / qmax).clamp(min=1e-12)
        zero = torch.zeros_like(scale)
        q = torch.clamp(torch.round(x / scale[..., None]), -qmax - 1, qmax)
    else:
        qmax = (1 << bits) - 1
        lo, hi = x.amin(dim=2), x.amax(dim=2)
        scale = ((hi - lo) / qmax).clamp(min=1e-12)
        zero = torch.round(-lo / scale)
        q = torch.clamp(torch.round(x / scale[..., None]) + zero[..., None], 0, qmax)
    w_hat = ((q - zero[..., None]) * scale[..., None]).view(out_f, -1)[:, :in_f]
    return w_hat, scale, zero


def naive_quantize(w: torch.Tensor, bits: int = 4, group_size: int = 128, symmetric: bool = True):
    return _group_quant(w.float(), bits, group_size, symmetric)[0]


# ------------------------------------------------------------------ GPTQ
@dataclass
class GptqConfig:
    bits: int = 4
    block_size: int = 128
    damp_percent: float = 0.01
    symmetric: bool = True
    group_size: int = 128


@dataclass
class GptqResult:
    quantized_weights: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    quantization_error: float
    bits: int


class GptqQuantizer:
    def __init__(self, config: GptqConfig | None = None):
        self.config = config or GptqConfig()

    @staticmethod
    def compute_hessian(x: torch.Tensor) -> torch.Tensor:
        x = x.double().reshape(-1, x.shape[-1])
        return 2.0 * x.t() @ x / max(1, x.shape[0])

    def _col_quant(self, col: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor):
        c = self.config
        if c.symmetric:
            qmax = (1 << (c.bits - 1)) - 1
            q = torch.clamp(torch.round(col / scale), -qmax - 1, qmax)
        else:
            qmax = (1 << c.bits) - 1
            q = torch.clamp(torch.round(col / scale) + zero, 0, qmax)
        return (q - zero) * scale

    def quantize(self, w: torch.Tensor, hessian: torch.Tensor) -> GptqResult:
        """w [out, in] (a Linear weight); hessian [in, in]."""
        c = self.config
        W = w.double().clone()
        out_f, in_f = W.shape
        H = hessian.double().clone()
        dead = torch.diag(H) == 0
        H[dead, dead] = 1.0
        W[:, dead] = 0.0
        H += torch.eye(in_f, dtype=H.dtype, device=H.device) * (c.damp_percent * torch.diag(H).mean())
        Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
        gs = in_f if c.group_size <= 0 else c.group_size
        Q = torch.zeros_like(W)
        scales, zeros = [], []
        scale = zero = None
        for b0 in range(0, in_f, c.block_size):
            b1 = min(in_f, b0 + c.block_size)
            W1 = W[:, b0:b1].clone()
            Err = torch.zeros_like(W1)
            Hb = Hinv[b0:b1, b0:b1]
            for i in range(b1 - b0):
                col_idx = b0 + i
                if col_idx % gs == 0:
                    _, s, z = _group_quant(W[:, col_idx : col_idx + gs].float(), c.bits, gs, c.symmetric)
                    scale, zero = s[:, 0].double(), z[:, 0].double()
                    scales.append(scale)
                    zeros.append(zero)
                col = W1[:, i]
                q = self._col_quant(col, scale, zero)
                Q[:, col_idx] = q
                e = (col - q) / Hb[i, i]
                W1[:, i:] -= e[:, None] * Hb[i, i:][None, :]
                Err[:, i] = e
            W[:, b0:b1] = W1
            W[:, b1:] -= Err @ Hinv[b0:b1, b1:]
        err = float(torch.linalg.norm(w.double() - Q))
        return GptqResult(Q.to(w.dtype), torch.stack(scales, 1).float(), torch.stack(zeros, 1).float(), err, c.bits)

    def quantize_with_calibration(self, w: torch.Tensor, calibration_inputs: torch.Tensor) -> GptqResult:
        return self.quantize(w, self.compute_hessian(calibration_inputs))


# ------------------------------------------------------------------ AWQ
@dataclass
class AwqConfig:
    bits: int = 4
    group_size: int = 128
    search_steps: int = 20
    zero_point: bool = False


class ActivationStats:
    def __init__(self, num_channels: int):
        self.sum = torch.zeros(num_channels, dtype=torch.float64)
        self.count = 0
        self.mean_abs = None

    def update(self, activations: torch.Tensor):
        a = activations.detach().reshape(-1, activations.shape[-1]).double().abs()
        self.sum = self.sum.to(a.device) + a.sum(0)
        self.count += a.shape[0]

    def finalize(self):
        self.mean_abs = self.sum / max(1, self.count)
        return self.mean_abs

    def num_channels(self) -> int:
        return self.sum.numel()


@dataclass
class AwqQuantizedLayer:
    weight: torch.Tensor  # quantize-dequantized, with the channel scale folded back
    scales: torch.Tensor  # per input channel
    alpha: float
    bits: int

    def dequantize_weights(self) -> torch.Tensor:
        return self.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.weight.t().to(x.dtype)

    def compression_ratio(self) -> float:
        return 32.0 / self.bits


class AwqQuantizer:
    def __init__(self, config: AwqConfig | None = None):
        self.config = config or AwqConfig()

    def find_optimal_scale(self, w: torch.Tensor, x: torch.Tensor, stats: torch.Tensor):
        c = self.config
        w, x, a = w.float(), x.float().reshape(-1, w.shape[1]), stats.float().to(w.device).clamp(min=1e-8)
        ref = x @ w.t()
        best = (float("inf"), 0.0, torch.ones_like(a))
        for i in range(c.search_steps):
            alpha = i / c.search_steps
            s = a.pow(alpha)
            s = s / (s.max() * s.min()).sqrt()
            wq = naive_quantize(w * s[None, :], c.bits, c.group_size, not c.zero_point) / s[None, :]
            err = float(((x @ wq.t() - ref) ** 2).mean())
            if err < best[0]:
                best = (err, alpha, s)
        return best[1], best[2]

    def quantize(self, w: torch.Tensor, calibration_inputs: torch.Tensor) -> AwqQuantizedLayer:
        st = ActivationStats(w.shape[1])
        st.update(calibration_inputs)
        alpha, s = self.find_optimal_scale(w, calibration_inputs, st.finalize())
        c = self.config
        wq = naive_quantize(w.float() * s[None, :], c.bits, c.group_size, not c.zero_point) / s[None, :]
        return AwqQuantizedLayer(wq, s, alpha, c.bits)


# ------------------------------------------------------------ SmoothQuant
@dataclass
class SmoothQuantConfig:
    alpha: float = 0.5
    bits: int = 8


def smooth_scales(act_absmax: torch.Tensor, w: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    wmax = w.float().abs().amax(dim=0).clamp(min=1e-5)
    return (act_absmax.float().clamp(min=1e-5).pow(alpha) / wmax.pow(1 - alpha)).clamp(min=1e-5)


def smooth_linear(x: torch.Tensor, w: torch.Tensor, alpha: float = 0.5):
    """Returns (x / s, w * s, s): the product is unchanged, the activation
    outliers are moved into the weights."""
    s = smooth_scales(x.reshape(-1, x.shape[-1]).abs().amax(0), w, alpha)
    return x / s, w * s[None, :], s


# ------------------------------------------------------------ observers
@dataclass
class ObserverStats:
    min_val: float = float("inf")
    max_val: float = float("-inf")
    count: int = 0


class Observer:
    def observe(self, t: torch.Tensor):
        raise NotImplementedError

    def stats(self) -> ObserverStats:
        return self._stats

    def reset(self):
        self._stats = ObserverStats()

    def compute_params(self, bits: int = 8, scheme=QuantizationScheme.SYMMETRIC) -> QuantizationParams:
        s = self.stats()
        return QuantizationParams.from_tensor(torch.tensor([s.min_val, s.max_val]), bits, scheme)


class MinMaxObserver(Observer):
    def __init__(self):
        self.reset()

    def observe(self, t: torch.Tensor):
        s = self._stats
        s.min_val = min(s.min_val, float(t.min()))
        s.max_val = max(s.max_val, float(t.max()))
        s.count += t.numel()


class PercentileObserver(Observer):
    def __init__(self, percentile: float = 99.99):
        if not 0.0 < percentile <= 100.0:
            raise ValueError("percentile must be in (0, 100]")
        self.percentile = percentile
        self._vals = []
        self.reset()

    def reset(self):
        self._stats = ObserverStats()
        self._vals = []

    def observe(self, t: torch.Tensor):
        self._vals.append(t.detach().float().reshape(-1).cpu())
        self._stats.count += t.numel()

    def finalize(self) -> ObserverStats:
        v = torch.cat(self._vals)
        q = self.percentile / 100.0
        self._stats.min_val = float(torch.quantile(v, 1 - q))
        self._stats.max_val = float(torch.quantile(v, q))
        return self._stats

    def stats(self) -> ObserverStats:
        return self.finalize() if self._vals else self._stats


class MovingAverageObserver(Observer):
    def __init__(self, alpha: float = 0.01):
        if not 0.0 < alpha <= 1.0:
            raise ValueError("alpha must be in (0, 1]")
        self.alpha = alpha
        self.reset()

    def observe(self, t: torch.Tensor):
        s = self._stats
        lo, hi = float(t.min()), float(t.max())
        if s.count == 0:
            s.min_val, s.max_val = lo, hi
        else:
            s.min_val += self.alpha * (lo - s.min_val)
            s.max_val += self.alpha * (hi - s.max_val)
        s.count += t.numel()


class CalibrationRunner:
    def __init__(self, factory=MinMaxObserver):
        self.factory = factory
        self.observers: dict[str, Observer] = {}

    def observe(self, name: str, t: torch.Tensor):
        self.observers.setdefault(name, self.factory()).observe(t)

    def all_stats(self) -> dict:
        return {k: o.stats() for k, o in self.observers.items()}

    def get_stats(self, name: str):
        o = self.observers.get(name)
        return o.stats() if o else None

    def get_observer(self, name: str):
        return self.observers.get(name)

    def reset_all(self):
        for o in self.observers.values():
            o.reset()


def minmax_calibration_runner() -> CalibrationRunner:
    return CalibrationRunner(MinMaxObserver)


class PostTrainingQuantizer:
    def __init__(self, config: QuantizationConfig | None = None):
        self.config = config or QuantizationConfig()
        self.runner = CalibrationRunner(MinMaxObserver)
        self.params: dict[str, QuantizationParams] = {}

    def add_calibration_data(self, name: str, t: torch.Tensor):
        self.runner.observe(name, t)

    def finalize_calibration(self) -> dict:
        c = self.config
        self.params = {k: o.compute_params(c.bits, c.scheme) for k, o in self.runner.observers.items()}
        return self.params

    def quantize_tensor(self, name: str, t: torch.Tensor) -> torch.Tensor:
        return self.params[name].quantize(t)


# ------------------------------------------------------------------ QAT
class FakeQuantLinear(nn.Module):
    """Linear layer whose weight (per tensor, symmetric) and input (running
    min/max, asymmetric) pass through fake quantization during training."""

    def __init__(self, linear: nn.Linear, bits: int = 8, momentum: float = 0.01):
        super().__init__()
        self.linear = linear
        self.bits = bits
        self.momentum = momentum
        self.register_buffer("act_min", torch.tensor(0.0))
        self.register_buffer("act_max", torch.tensor(0.0))
        self.register_buffer("seen", torch.tensor(0))

    def forward(self, x):
        if self.training:
            lo, hi = x.detach().min(), x.detach().max()
            if int(self.seen) == 0:
                self.act_min.copy_(lo)
                self.act_max.copy_(hi)
            else:
                self.act_min += self.momentum * (lo - self.act_min)
                self.act_max += self.momentum * (hi - self.act_max)
            self.seen += 1
        lo, hi = min(float(self.act_min), 0.0), max(float(self.act_max), 0.0)
        qmax_u = (1 << self.bits) - 1
        if hi > lo:
            sa = (hi - lo) / qmax_u
            x = fake_quantize(x, sa, int(round(-lo / sa)), 0, qmax_u)
        qm = (1 << (self.bits - 1)) - 1
        w = self.linear.weight
        sw = float(w.detach().abs().max()) / qm or 1.0
        wq = fake_quantize(w, sw, 0, -qm, qm)
        return nn.functional.linear(x, wq, self.linear.bias)


class QuantizationAwareTraining:
    """Swap every nn.Linear of a module for a FakeQuantLinear."""

    def __init__(self, bits: int = 8):
        self.bits = bits

    def prepare(self, module: nn.Module) -> nn.Module:
        for name, child in list(module.named_children()):
            if isinstance(child, nn.Linear):
                setattr(module, name, FakeQuantLinear(child, self.bits))
            else:
                self.prepare(child)
        return module
