"""Integer quantization primitives: int8 (symmetric / asymmetric, per
tensor / per output channel), int4 groups packed two per byte, generic
n-bit affine parameters, and quantized matmul.

Reference parity: scirs2-neural/src/quantization/int8.rs:11-300 (Int8Mode,
Granularity, Int8Params, Int8Tensor, quantize_int8, dequantize_int8,
quantized_matmul, roundtrip_mse), int4.rs:12-240 (GroupSize, Int4Tensor,
quantize_int4 / dequantize_int4 with low nibble = even element),
mod.rs:26-230 (QuantizationConfig / Scheme / Mode / Params, QuantizedTensor).
The rules (scale = amax / 127; asymmetric range 255 with a zero point;
int4 scale = (max - min) / 15, zero point in 0..15) are the definitions of
these formats.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

import torch


class Int8Mode(enum.Enum):
    SYMMETRIC = "symmetric"
    ASYMMETRIC = "asymmetric"


class Granularity(enum.Enum):
    PER_TENSOR = "per_tensor"
    PER_CHANNEL = "per_channel"


@dataclass
class Int8Tensor:
    data: torch.Tensor        # int8, original shape
    scale: torch.Tensor       # fp32 [channels] (1 for per-tensor)
    zero_point: torch.Tensor  # int32 [channels]
    granularity: Granularity
    mode: Int8Mode

    @property
    def shape(self):
        return tuple(self.data.shape)

    def size_bytes(self) -> int:
        return self.data.numel() + 8 * self.scale.numel()


def _channels(t: torch.Tensor, gran: Granularity) -> torch.Tensor:
    return t.reshape(1, -1) if gran == Granularity.PER_TENSOR else t.reshape(t.shape[0], -1)


def quantize_int8(t: torch.Tensor, mode: Int8Mode = Int8Mode.SYMMETRIC,
                  granularity: Granularity = Granularity.PER_TENSOR) -> Int8Tensor:
    x = _channels(t.float(), granularity)
    if mode == Int8Mode.SYMMETRIC:
        amax = x.abs().amax(dim=1)
        scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
        zp = torch.zeros_like(scale, dtype=torch.int32)
        q = torch.clamp(torch.round(x / scale[:, None]), -127, 127)
    else:
        lo = torch.clamp(x.amin(dim=1), max=0.0)
        hi = torch.clamp(x.amax(dim=1), min=0.0)
        scale = torch.where(hi > lo, (hi - lo) / 255.0, torch.ones_like(hi))
        zp = (torch.round(-lo / scale) - 128).to(torch.int32)
        q = torch.clamp(torch.round(x / scale[:, None]) + zp[:, None], -128, 127)
    return Int8Tensor(q.to(torch.int8).reshape(t.shape), scale, zp, granularity, mode)


def dequantize_int8(q: Int8Tensor) -> torch.Tensor:
    x = _channels(q.data.float(), q.granularity)
    return ((x - q.zero_point[:, None].float()) * q.scale[:, None]).reshape(q.data.shape)


def roundtrip_mse(t: torch.Tensor, mode=Int8Mode.SYMMETRIC, granularity=Granularity.PER_TENSOR) -> float:
    return float(((dequantize_int8(quantize_int8(t, mode, granularity)) - t.float()) ** 2).mean())


def quantized_matmul(a: torch.Tensor, b: torch.Tensor, mode: Int8Mode = Int8Mode.SYMMETRIC) -> torch.Tensor:
    """a [M, K] @ b [K, N] through int8 per-tensor quantization of both
    operands: integer products accumulated exactly, then rescaled."""
    qa, qb = quantize_int8(a, mode), quantize_int8(b, mode)
    ia = qa.data.to(torch.int64) - qa.zero_point[0]
    ib = qb.data.to(torch.int64) - qb.zero_point[0]
    if ia.is_cuda:  # exact in fp64 for |products| < 2^53
        acc = ia.double() @ ib.double()
    else:
        acc = (ia @ ib).double()
    return (acc * (float(qa.scale[0]) * float(qb.scale[0]))).float()


class GroupSize(enum.IntEnum):
    G32 = 32
    G64 = 64
    G128 = 128


@dataclass
class Int4Tensor:
    packed: torch.Tensor      # uint8 [ceil(n/2)], low nibble = even element
    scale: torch.Tensor       # fp32 [groups]
    zero_point: torch.Tensor  # uint8 [groups] in 0..15
    group_size: int
    shape: tuple
    n_elements: int

    def memory_bytes(self) -> int:
        return self.packed.numel() + self.scale.numel() * 4 + self.zero_point.numel()

    def compression_ratio(self) -> float:
        return self.n_elements * 4 / self.memory_bytes()


def quantize_int4(t: torch.Tensor, group_size: int = GroupSize.G128) -> Int4Tensor:
    gs = int(group_size)
    flat = t.float().reshape(-1)
    n = flat.numel()
    pad = (-n) % gs
    x = torch.cat([flat, flat.new_zeros(pad)]).view(-1, gs)
    lo, hi = x.amin(dim=1), x.amax(dim=1)
    scale = torch.where(hi > lo, (hi - lo) / 15.0, torch.ones_like(hi))
    zp = torch.clamp(torch.round(-lo / scale), 0, 15)
    q = torch.clamp(torch.round(x / scale[:, None]) + zp[:, None], 0, 15).to(torch.uint8).reshape(-1)[:n]
    if n % 2:
        q = torch.cat([q, q.new_zeros(1)])
    packed = (q[0::2] | (q[1::2] << 4)).to(torch.uint8)
    return Int4Tensor(packed, scale, zp.to(torch.uint8), gs, tuple(t.shape), n)


def dequantize_int4(q: Int4Tensor) -> torch.Tensor:
    lo = (q.packed & 0x0F).to(torch.float32)
    hi = (q.packed >> 4).to(torch.float32)
    vals = torch.stack([lo, hi], dim=1).reshape(-1)[: q.n_elements]
    g = torch.arange(q.n_elements, device=vals.device) // q.group_size
    return ((vals - q.zero_point.float()[g]) * q.scale[g]).reshape(q.shape)


def int4_roundtrip_mse(t: torch.Tensor, group_size: int = GroupSize.G128) -> float:
    return float(((dequantize_int4(quantize_int4(t, group_size)) - t.float()) ** 2).mean())


# ---------------------------------------------------------------------------
# generic n-bit affine quantization
# ---------------------------------------------------------------------------
class QuantizationScheme(enum.Enum):
    SYMMETRIC = "symmetric"
    ASYMMETRIC = "asymmetric"


class QuantizationMode(enum.Enum):
    DYNAMIC = "dynamic"
    STATIC = "static"
    QAT = "qat"


@dataclass
class QuantizationConfig:
    bits: int = 8
    scheme: QuantizationScheme = QuantizationScheme.SYMMETRIC
    mode: QuantizationMode = QuantizationMode.STATIC
    per_channel: bool = False
    calibration_samples: int = 100


@dataclass
class QuantizationParams:
    bits: int = 8
    signed: bool = True
    scale: float = 1.0
    zero_point: int = 0
    qmin: int = field(default=-128)
    qmax: int = field(default=127)

    @staticmethod
    def new(bits: int, signed: bool) -> "QuantizationParams":
        qmin, qmax = (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if signed else (0, (1 << bits) - 1)
        return QuantizationParams(bits, signed, 1.0, 0, qmin, qmax)

    @staticmethod
    def from_tensor(t: torch.Tensor, bits: int, scheme: QuantizationScheme) -> "QuantizationParams":
        p = QuantizationParams.new(bits, scheme == QuantizationScheme.SYMMETRIC)
        if scheme == QuantizationScheme.SYMMETRIC:
            amax = float(t.abs().max()) if t.numel() else 0.0
            p.scale = amax / p.qmax if amax > 0 else 1.0
        else:
            lo, hi = min(float(t.min()), 0.0), max(float(t.max()), 0.0)
            p.scale = (hi - lo) / (p.qmax - p.qmin) if hi > lo else 1.0
            p.zero_point = int(round(p.qmin - lo / p.scale))
        return p

    def quantize(self, t: torch.Tensor) -> torch.Tensor:
        return torch.clamp(torch.round(t.float() / self.scale) + self.zero_point, self.qmin, self.qmax)

    def dequantize(self, q: torch.Tensor) -> torch.Tensor:
        return (q.float() - self.zero_point) * self.scale


@dataclass
class QuantizedTensor:
    data: torch.Tensor
    params: QuantizationParams
    shape: tuple

    @staticmethod
    def from_float(t: torch.Tensor, config: QuantizationConfig) -> "QuantizedTensor":
        p = QuantizationParams.from_tensor(t, config.bits, config.scheme)
        dt = torch.int8 if config.bits <= 8 and p.signed else (torch.uint8 if config.bits <= 8 else torch.int32)
        return QuantizedTensor(p.quantize(t).to(dt), p, tuple(t.shape))

    def dequantize(self) -> torch.Tensor:
        return self.params.dequantize(self.data)

    def size_bytes(self) -> int:
        return (self.data.numel() * self.params.bits + 7) // 8

    def compression_ratio(self) -> float:
        return self.data.numel() * 4 / max(1, self.size_bytes())


def fake_quantize(t: torch.Tensor, scale: float, zero_point: int, qmin: int, qmax: int) -> torch.Tensor:
    """Quantize-dequantize with a straight-through gradient inside the range."""
    return _FakeQuant.apply(t, scale, zero_point, qmin, qmax)


class _FakeQuant(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, zp, qmin, qmax):
        q = torch.round(x / scale) + zp
        ctx.save_for_backward((q >= qmin) & (q <= qmax))
        return (torch.clamp(q, qmin, qmax) - zp) * scale

    @staticmethod
    def backward(ctx, g):
        (inside,) = ctx.saved_tensors
        return g * inside, None, None, None, None
