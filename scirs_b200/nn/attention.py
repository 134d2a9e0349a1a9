"""Attention layers and positional schemes.

  MultiHeadAttention / SelfAttention   scirs2-neural/src/layers/attention.rs:29-658
  FlashAttentionV2 (+config, compute)  scirs2-neural/src/layers/flash_attention_v2.rs:23-520
  RopeEmbedding                        scirs2-neural/src/attention/rope.rs:53-250
  AlibiSlopes                          scirs2-neural/src/attention/alibi.rs:45-190
  SlidingWindowAttention               scirs2-neural/src/attention/sliding_window.rs:39-219
  SparseAttention (masks)              scirs2-neural/src/attention/sparse/attention.rs:40-218
  GroupedQueryAttention / MQA + KvCache scirs2-neural/src/layers/grouped_query_attention.rs:71-589

The reference computes these forward-only on the CPU (backward is an
identity stub or NotImplemented there). Here they are differentiable; the
dense causal / non-causal case with head_dim 64 or 128 in bf16 on CUDA runs
on the framework's flash-attention kernels; masks and biases use PyTorch.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import functional as FN
from .base import Layer


@dataclass
class AttentionConfig:
    num_heads: int = 8
    head_dim: int = 64
    dropout_prob: float = 0.0
    causal: bool = False
    scale: float | None = None


def _uniform_proj(d_in, d_out, g, dtype, device):
    bound = math.sqrt(6.0 / (d_in + d_out))  # Xavier uniform
    return nn.Parameter(((torch.rand(d_in, d_out, generator=g) * 2 - 1) * bound).to(dtype=dtype, device=device))


class MultiHeadAttention(Layer):
    """Projections W_q, W_k, W_v, W_o of shape [d_model, d_model], no bias
    (parameter_count = 4 d^2, as the reference), scaled dot-product attention
    per head with an optional causal mask. Input [B, S, d_model]."""

    def __init__(self, d_model: int, config: AttentionConfig | None = None, *, seed: int | None = None,
                 dtype=torch.float32, device=None):
        super().__init__()
        self.config = config or AttentionConfig(num_heads=8, head_dim=d_model // 8)
        c = self.config
        if c.num_heads * c.head_dim != d_model:
            raise ValueError("num_heads * head_dim must equal d_model")
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        self.d_model = d_model
        self.w_query = _uniform_proj(d_model, d_model, g, dtype, device)
        self.w_key = _uniform_proj(d_model, d_model, g, dtype, device)
        self.w_value = _uniform_proj(d_model, d_model, g, dtype, device)
        self.w_output = _uniform_proj(d_model, d_model, g, dtype, device)

    def _attend(self, q, k, v):
        c = self.config
        scale = c.scale if c.scale is not None else c.head_dim**-0.5
        o = FN.attention(q, k, v, causal=c.causal, scale=scale)
        if c.dropout_prob > 0 and self.training:
            o = F.dropout(o, c.dropout_prob)
        return o

    def forward(self, x, key_value: torch.Tensor | None = None):
        B, S, D = x.shape
        c = self.config
        kv = x if key_value is None else key_value
        q = FN.linear(x, self.w_query).view(B, S, c.num_heads, c.head_dim)
        k = FN.linear(kv, self.w_key).view(B, kv.shape[1], c.num_heads, c.head_dim)
        v = FN.linear(kv, self.w_value).view(B, kv.shape[1], c.num_heads, c.head_dim)
        o = self._attend(q, k, v).reshape(B, S, D)
        return FN.linear(o, self.w_output)


class SelfAttention(MultiHeadAttention):
    """Multi-head self-attention (query = key = value = input)."""

    def forward(self, x):
        return super().forward(x)


@dataclass
class FlashAttentionV2Config:
    num_heads: int = 8
    head_dim: int = 64
    block_size_q: int = 128
    block_size_kv: int = 128
    causal: bool = False
    dropout_prob: float = 0.0
    scale: float | None = None

    def with_block_size_q(self, b):
        self.block_size_q = b
        return self

    def with_block_size_kv(self, b):
        self.block_size_kv = b
        return self

    def with_causal(self, c):
        self.causal = c
        return self

    def with_dropout(self, p):
        self.dropout_prob = p
        return self

    def with_scale(self, s):
        self.scale = s
        return self


class FlashAttentionV2(MultiHeadAttention):
    """Attention layer with projections whose core is the tiled online-softmax
    kernel (blocks are chosen by the kernel; the config's block sizes are
    kept for API parity and used by :func:`flash_attention_v2_compute`)."""

    def __init__(self, d_model: int, config: FlashAttentionV2Config, *, seed=None, dtype=torch.float32, device=None):
        self.fa_config = config
        super().__init__(
            d_model,
            AttentionConfig(config.num_heads, config.head_dim, config.dropout_prob, config.causal, config.scale),
            seed=seed,
            dtype=dtype,
            device=device,
        )


def flash_attention_v2_compute(q, k, v, causal: bool = False, block_q: int = 128, block_kv: int = 128,
                               scale: float | None = None):
    """Blocked online-softmax attention on [S, d] (single head) or [B, S, H, d]
    tensors. On bf16 CUDA tensors this is the framework kernel; otherwise the
    tiled algorithm runs in PyTorch with the given block sizes (this is the
    reference's CPU algorithm, scirs2-neural/src/attention/flash_v2.rs:96-300)."""
    single = q.dim() == 2
    if single:
        q, k, v = (t[None, :, None, :] for t in (q, k, v))
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    if q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] in (64, 128):
        o = FN.attention(q, k, v, causal=causal, scale=scale)
    else:
        B, S, H, D = q.shape
        qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
        o = torch.zeros_like(qf)
        for i0 in range(0, S, block_q):
            qi = qf[:, :, i0 : i0 + block_q]
            m = torch.full(qi.shape[:-1], float("-inf"), device=q.device)
            l = torch.zeros_like(m)
            acc = torch.zeros_like(qi)
            for j0 in range(0, kf.shape[2], block_kv):
                if causal and j0 > i0 + qi.shape[2] - 1:
                    break
                s = qi @ kf[:, :, j0 : j0 + block_kv].transpose(-1, -2) * scale
                if causal:
                    qi_idx = torch.arange(i0, i0 + qi.shape[2], device=q.device)[:, None]
                    kj_idx = torch.arange(j0, j0 + s.shape[-1], device=q.device)[None, :]
                    s = s.masked_fill(kj_idx > qi_idx, float("-inf"))
                mn = torch.maximum(m, s.amax(-1))
                p = torch.exp(s - mn[..., None])
                alpha = torch.exp(m - mn)
                l = l * alpha + p.sum(-1)
                acc = acc * alpha[..., None] + p @ vf[:, :, j0 : j0 + block_kv]
                m = mn
            o[:, :, i0 : i0 + block_q] = acc / l[..., None]
        o = o.transpose(1, 2).to(q.dtype)
    return o[0, :, 0, :] if single else o


# ---------------------------------------------------------------------------- RoPE
@dataclass
class RopeConfig:
    base: float = 10000.0
    dim: int = 0
    max_seq_len: int = 4096


class RopeEmbedding:
    """Rotary position embedding, half-rotation (NeoX) form:
    (x_i, x_{i+d/2}) -> (x_i cos - x_{i+d/2} sin, x_i sin + x_{i+d/2} cos),
    theta_i = base^(-2i/d)."""

    def __init__(self, config: RopeConfig):
        self.config = config
        d = config.dim
        half = d // 2
        inv = config.base ** (-2.0 * torch.arange(half, dtype=torch.float64) / max(d, 1))
        ang = torch.arange(config.max_seq_len, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos_table = torch.cos(ang).float()
        self.sin_table = torch.sin(ang).float()

    def apply(self, x: torch.Tensor, offset: int = 0) -> torch.Tensor:
        """x: [..., S, H, head_dim] or [..., S, head_dim]; rotates the first
        `dim` features of every head; returns a new tensor."""
        d = min(self.config.dim, x.shape[-1])
        if d == 0 or d % 2:
            return x
        S = x.shape[-3] if x.dim() >= 3 else x.shape[-2]
        cos = self.cos_table[offset : offset + S].to(x.device)
        sin = self.sin_table[offset : offset + S].to(x.device)
        if x.dim() >= 3:
            cos, sin = cos[:, None, :], sin[:, None, :]
        half = d // 2
        x1, x2, rest = x[..., :half].float(), x[..., half:d].float(), x[..., d:]
        out = torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1).to(x.dtype)
        return torch.cat([out, rest], -1) if rest.shape[-1] else out

    def cos_at(self, m):
        return self.cos_table[m]

    def sin_at(self, m):
        return self.sin_table[m]

    def base(self):
        return self.config.base

    def dim(self):
        return self.config.dim

    def table_len(self):
        return self.cos_table.shape[0]


# ---------------------------------------------------------------------------- ALiBi
@dataclass
class AlibiConfig:
    num_heads: int = 8


class AlibiSlopes:
    """Linear-bias slopes m_h = 2^(-8h/H), bias[i,j] = -m_h |i-j|."""

    def __init__(self, config: AlibiConfig):
        self.config = config
        self._slopes = self.compute_slopes(config.num_heads)

    @staticmethod
    def compute_slopes(num_heads: int) -> list[float]:
        return [2.0 ** (-8.0 * h / num_heads) for h in range(1, num_heads + 1)]

    def slopes(self):
        return list(self._slopes)

    def slope_at(self, h):
        return self._slopes[h] if 0 <= h < len(self._slopes) else None

    def get_bias_matrix(self, seq_len: int, device=None) -> torch.Tensor:
        i = torch.arange(seq_len, device=device)
        dist = (i[:, None] - i[None, :]).abs().float()
        s = torch.tensor(self._slopes, device=device)[:, None, None]
        return -s * dist

    def apply_to_attention_scores(self, scores: torch.Tensor) -> torch.Tensor:
        """scores [..., H, S, S] -> scores + bias."""
        return scores + self.get_bias_matrix(scores.shape[-1], scores.device).to(scores.dtype)


def attention_with_bias(q, k, v, bias=None, mask=None, scale=None):
    """Reference attention with an additive bias [H,S,S] and/or boolean keep
    mask [S,S] on [B, S, H, D] tensors (differentiable)."""
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) * scale
    if bias is not None:
        s = s + bias.float()
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, -1)
    return torch.einsum("bhqk,bkhd->bqhd", p, v.float()).to(q.dtype)


# ---------------------------------------------------------------------------- sliding window / sparse
@dataclass
class SlidingWindowConfig:
    window_size: int = 512
    global_tokens: int = 0


class SlidingWindowAttention:
    """Token i attends to [i-w, i+w] plus `global_tokens` leading tokens that
    attend everywhere and are attended by everyone. On CUDA (bf16, head_dim
    64 / 128) the kernels visit only the key blocks the window touches
    (ops.sparse_attention); no S x S mask is built."""

    def __init__(self, config: SlidingWindowConfig, causal: bool = False):
        self.config = config
        self.causal = causal

    def pattern(self):
        from ..ops.sparse_attention import sliding_window

        return sliding_window(self.config.window_size, self.config.global_tokens, self.causal)

    def mask(self, S: int, device=None) -> torch.Tensor:
        """Dense [S, S] mask of the pattern (for inspection and the CPU path)."""
        return self.pattern().allowed_dense(S, S, device=device)

    def forward(self, q, k, v, scale=None):
        if q.is_cuda:
            plan = self.pattern().plan(q.shape[1], k.shape[1], q.shape[-1], q.device)
            return FN.attention(q, k, v, False, scale, plan=plan)
        return attention_with_bias(q, k, v, mask=self.mask(q.shape[1], q.device), scale=scale)


class SparseAttention:
    """Attention restricted to a sparse pattern.

    Block patterns (run on the sparse kernels on CUDA, no dense mask):
      'block_strided'  Sparse-Transformer layout over 128-token blocks: the
                       `local` nearest key blocks plus every `block_stride`-th block
      'bigbird'        window of `window` tokens + `num_global` global tokens
                       + `num_random` random key blocks per query block
      bitmap=          any [q blocks, k blocks] boolean layout of 128 x 128 blocks
    Token patterns (dense mask, evaluated with the masked reference):
      'strided' (local band + every stride-th column), 'fixed' (block-local +
      summary columns) or a user `mask`."""

    def __init__(self, pattern: str = "strided", stride: int = 64, block: int = 64, mask: torch.Tensor | None = None,
                 local: int = 1, window: int = 128, num_global: int = 0, num_random: int = 2, seed: int = 0,
                 causal: bool = False, bitmap: torch.Tensor | None = None, block_stride: int = 4):
        self.pattern, self.stride, self.block, self.user_mask = pattern, stride, block, mask
        self.local, self.window, self.num_global, self.num_random = local, window, num_global, num_random
        self.seed, self.causal, self.bitmap, self.block_stride = seed, causal, bitmap, block_stride

    def block_pattern(self, Sq: int, Sk: int):
        """The AttentionPattern of a block pattern (None for token patterns)."""
        from ..ops import sparse_attention as SA

        nq, nk = (Sq + 127) // 128, (Sk + 127) // 128
        if self.bitmap is not None:
            return SA.block_sparse(self.bitmap, causal=self.causal)
        if self.pattern == "block_strided":
            bm = SA.strided_bitmap(nq, nk, self.local, self.block_stride, self.causal)
            return SA.block_sparse(bm, causal=self.causal, key=f"strided{nq}x{nk}:{self.local}:{self.block_stride}")
        if self.pattern == "bigbird":
            g = torch.Generator().manual_seed(self.seed)
            bm = torch.zeros(nq, nk, dtype=torch.bool)
            for i in range(nq):
                bm[i, torch.randperm(nk, generator=g)[: self.num_random]] = True
            return SA.AttentionPattern(causal=self.causal, window_left=self.window, num_global=self.num_global,
                                       bitmap=bm, bitmap_key=f"bigbird{nq}x{nk}:{self.num_random}:{self.seed}")
        return None

    def mask(self, S: int, device=None) -> torch.Tensor:
        if self.user_mask is not None:
            return self.user_mask.to(device)
        bp = self.block_pattern(S, S)
        if bp is not None:
            return bp.allowed_dense(S, S, device=device)
        i = torch.arange(S, device=device)
        if self.pattern == "strided":
            local = (i[:, None] - i[None, :]).abs() < self.stride
            strided = (i[None, :] % self.stride) == (self.stride - 1)
            return local | strided
        blk = (i[:, None] // self.block) == (i[None, :] // self.block)
        summary = (i[None, :] % self.block) == (self.block - 1)
        return blk | summary

    def forward(self, q, k, v, scale=None):
        bp = self.block_pattern(q.shape[1], k.shape[1]) if self.user_mask is None else None
        if bp is not None and q.is_cuda:
            return FN.attention(q, k, v, False, scale, plan=bp.plan(q.shape[1], k.shape[1], q.shape[-1], q.device))
        return attention_with_bias(q, k, v, mask=self.mask(q.shape[1], q.device), scale=scale)


# ---------------------------------------------------------------------------- GQA / MQA
class KvCache:
    """Append-only key/value cache for incremental decoding [B, S, Hkv, D]."""

    def __init__(self):
        self.k = None
        self.v = None

    def append(self, k, v):
        self.k = k if self.k is None else torch.cat([self.k, k], 1)
        self.v = v if self.v is None else torch.cat([self.v, v], 1)
        return self.k, self.v

    def __len__(self):
        return 0 if self.k is None else self.k.shape[1]

    def clear(self):
        self.k = self.v = None


class GroupedQueryAttention(Layer):
    """num_heads query heads share num_kv_heads key/value heads (MQA when
    num_kv_heads == 1). Optional RoPE, causal mask and KV cache."""

    def __init__(self, d_model: int, num_heads: int, num_kv_heads: int, *, causal: bool = True,
                 rope: RopeEmbedding | None = None, seed=None, dtype=torch.float32, device=None):
        super().__init__()
        if num_heads % num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.h, self.hkv, self.hd = num_heads, num_kv_heads, d_model // num_heads
        self.causal, self.rope = causal, rope
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        self.w_q = _uniform_proj(d_model, d_model, g, dtype, device)
        self.w_k = _uniform_proj(d_model, self.hkv * self.hd, g, dtype, device)
        self.w_v = _uniform_proj(d_model, self.hkv * self.hd, g, dtype, device)
        self.w_o = _uniform_proj(d_model, d_model, g, dtype, device)

    def forward(self, x, cache: KvCache | None = None):
        return self.forward_with_cache(x, cache)

    def forward_with_cache(self, x, cache: KvCache | None = None):
        B, S, D = x.shape
        off = len(cache) if cache is not None else 0
        q = FN.linear(x, self.w_q).view(B, S, self.h, self.hd)
        k = FN.linear(x, self.w_k).view(B, S, self.hkv, self.hd)
        v = FN.linear(x, self.w_v).view(B, S, self.hkv, self.hd)
        if self.rope is not None:
            q, k = self.rope.apply(q, off), self.rope.apply(k, off)
        if cache is not None:
            k, v = cache.append(k, v)
        rep = self.h // self.hkv
        if rep > 1:
            k = k.repeat_interleave(rep, dim=2)
            v = v.repeat_interleave(rep, dim=2)
        if off == 0 and k.shape[1] == S:
            o = FN.attention(q, k, v, causal=self.causal)
        else:  # decoding against a cache: query positions are off..off+S-1
            Sk = k.shape[1]
            qi = torch.arange(off, off + S, device=x.device)[:, None]
            kj = torch.arange(Sk, device=x.device)[None, :]
            o = attention_with_bias(q, k, v, mask=(kj <= qi) if self.causal else None)
        return FN.linear(o.reshape(B, S, D), self.w_o)


class MultiQueryAttention(GroupedQueryAttention):
    def __init__(self, d_model: int, num_heads: int, **kw):
        super().__init__(d_model, num_heads, 1, **kw)
