"""Functional attention on [batch, seq, d_model] tensors (one head unless a
projection / head count says otherwise).

Every function is differentiable and runs on any device. Where the math is
plain softmax attention (no mask, or a causal one) on CUDA bf16 tensors with
head_dim 64 or 128, it runs on the framework's tcgen05 flash-attention kernels
through `ops.functional.attention`; the projections of `multi_head_attention`
and `grouped_query_attention` run on the framework's GEMM through
`ops.functional.linear` under the same conditions. Everything else is
PyTorch math. Shapes, argument order and edge cases follow the reference's
functional attention module so that code written against it ports directly:

* masks: additive (added to the scores), multiplicative (multiplied into the
  probabilities after the softmax), boolean (False = not attended) or causal;
  mask tensors are [B or 1, Lq, Lk];
* a row with no attended key gives a zero output row (sparse attention);
* ALiBi on these single-head tensors applies the first slope, bias
  -slope * |i - j|, then the optional causal mask;
* RoPE rotates interleaved pairs (2i, 2i + 1) by pos * base^(-2i / d);
* linear attention maps q and (scale * k) through elu(x) + 1 and divides by the
  normaliser q' . sum_k k' (rows with a non-positive normaliser give zeros); the
  reference documents this feature map but its code returns x, not x + 1, for
  x > 0 (a map that jumps from 1 to 0 at x = 0); this module uses elu(x) + 1;
* relative-position attention adds q . rel_emb[(Lk - 1) + i - j] to q . k_j,
  both times `scale`, with rel_emb of shape [2 max(Lq, Lk) - 1, d];
* xPos scales q and k at 1-based position p by p^(-j / d) along the feature j.

Reference parity: scirs2-linalg/src/attention/scaled_dot_product.rs:32-230,
cross_attention.rs:32-820 (flash, sparse, ALiBi, rotary, linear,
relative-position, RPE / xPos), multi_head.rs:36-330 (multi-head and
grouped-query attention), utils.rs:14-49 (AttentionMask, AttentionConfig).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

_KINDS = ("additive", "multiplicative", "boolean", "causal")


@dataclass
class AttentionMask:
    """`kind` is one of additive / multiplicative / boolean / causal; `tensor`
    ([B or 1, Lq, Lk]) is unused for causal."""

    kind: str
    tensor: torch.Tensor | None = None

    def __post_init__(self):
        if self.kind not in _KINDS:
            raise ValueError(f"mask kind must be one of {_KINDS}, got {self.kind!r}")
        if self.kind != "causal" and self.tensor is None:
            raise ValueError(f"a {self.kind} mask needs a tensor")

    @staticmethod
    def additive(t):
        return AttentionMask("additive", t)

    @staticmethod
    def multiplicative(t):
        return AttentionMask("multiplicative", t)

    @staticmethod
    def boolean(t):
        return AttentionMask("boolean", t)

    @staticmethod
    def causal():
        return AttentionMask("causal")


@dataclass
class AttentionConfig:
    num_heads: int
    head_dim: int
    dropout_prob: float = 0.0
    causal: bool = False
    scale: float | None = None


def _check3(q, k, v):
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("query, key and value must be [batch, seq, d_model]")
    if not (q.shape[0] == k.shape[0] == v.shape[0]):
        raise ValueError(f"batch sizes must match: {q.shape[0]}, {k.shape[0]}, {v.shape[0]}")
    if k.shape[1] != v.shape[1]:
        raise ValueError(f"key and value sequence lengths must match: {k.shape[1]}, {v.shape[1]}")
    if q.shape[2] != k.shape[2]:
        raise ValueError(f"query and key dimensions must match: {q.shape[2]}, {k.shape[2]}")


def _kernel_ok(q, k, v, causal):
    return (q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == v.dtype == torch.bfloat16
            and q.shape[-1] in (64, 128) and v.shape[-1] == q.shape[-1]
            and (not causal or q.shape[-2] == k.shape[-2]))


def _heads_attention(q, k, v, causal, scale):
    """q [B, Lq, H, D], k / v [B, Lk, H, D] -> [B, Lq, H, D]."""
    from ..ops import functional as OF

    if _kernel_ok(q, k, v, causal):
        return OF.attention(q, k, v, causal=causal, scale=scale)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                       is_causal=causal, scale=scale)
    return o.transpose(1, 2)


def _scores_attention(q, k, v, scale, mask: AttentionMask | None, causal: bool = False):
    """Dense reference path with every mask kind (and an optional causal mask on top)."""
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    Lq, Lk = s.shape[-2], s.shape[-1]
    if causal and (mask is None or mask.kind != "causal"):
        tri = torch.ones(Lq, Lk, dtype=torch.bool, device=s.device).tril()
        s = s.masked_fill(~tri, float("-inf"))
    if mask is not None:
        if mask.kind == "causal":
            tri = torch.ones(Lq, Lk, dtype=torch.bool, device=s.device).tril()
            s = s.masked_fill(~tri, float("-inf"))
        elif mask.kind == "additive":
            s = s + mask.tensor.to(s.dtype)
        elif mask.kind == "boolean":
            s = s.masked_fill(~mask.tensor.to(torch.bool), float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)  # fully masked rows
    if mask is not None and mask.kind == "multiplicative":
        p = p * mask.tensor.to(p.dtype)
    return torch.matmul(p, v)


def scaled_dot_product_attention(query, key, value, mask: AttentionMask | None = None, scale: float | None = None):
    """softmax(scale q k^T [+ mask]) v on [B, L, d] tensors."""
    _check3(query, key, value)
    scale = scale if scale is not None else query.shape[-1] ** -0.5
    if mask is None or mask.kind == "causal":
        causal = mask is not None
        if _kernel_ok(query, key, value, causal):
            return _heads_attention(query.unsqueeze(2), key.unsqueeze(2), value.unsqueeze(2), causal,
                                    scale).squeeze(2)
    return _scores_attention(query, key, value, scale, mask)


def masked_attention(query, key, value, mask: AttentionMask, scale: float | None = None):
    return scaled_dot_product_attention(query, key, value, mask, scale)


def causal_attention(query, key, value, scale: float | None = None):
    return scaled_dot_product_attention(query, key, value, AttentionMask.causal(), scale)


def flash_attention(query, key, value, mask: AttentionMask | None = None, scale: float | None = None,
                    block_size: int = 64):
    """Same result as scaled_dot_product_attention, computed tile by tile over the keys with an online
    softmax (block_size keys per tile) when it does not run on the flash kernels."""
    _check3(query, key, value)
    scale = scale if scale is not None else query.shape[-1] ** -0.5
    if mask is None or mask.kind == "causal":
        causal = mask is not None
        if _kernel_ok(query, key, value, causal):
            return scaled_dot_product_attention(query, key, value, mask, scale)
    if mask is not None and mask.kind == "multiplicative":
        return _scores_attention(query, key, value, scale, mask)  # needs the normalised probabilities
    if block_size < 1:
        raise ValueError("block_size must be positive")
    B, Lq, _ = query.shape
    Lk = key.shape[1]
    ct = torch.float64 if query.dtype == torch.float64 else torch.float32  # accumulate in >= fp32
    qf, kf, vf = query.to(ct), key.to(ct), value.to(ct)
    m = torch.full((B, Lq, 1), float("-inf"), device=query.device, dtype=ct)
    den = torch.zeros(B, Lq, 1, device=query.device, dtype=ct)
    acc = torch.zeros(B, Lq, value.shape[-1], device=query.device, dtype=ct)
    rows = torch.arange(Lq, device=query.device)[:, None]
    for j0 in range(0, Lk, block_size):
        j1 = min(Lk, j0 + block_size)
        s = torch.matmul(qf, kf[:, j0:j1].transpose(-1, -2)) * scale
        if mask is not None:
            if mask.kind == "causal":
                cols = torch.arange(j0, j1, device=query.device)[None, :]
                s = s.masked_fill(cols > rows, float("-inf"))
            elif mask.kind == "additive":
                s = s + mask.tensor[..., j0:j1].to(ct)
            elif mask.kind == "boolean":
                s = s.masked_fill(~mask.tensor[..., j0:j1].to(torch.bool), float("-inf"))
        m_new = torch.maximum(m, s.amax(-1, keepdim=True))
        safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
        alpha = torch.exp(m - safe)
        p = torch.exp(s - safe)
        den = den * alpha + p.sum(-1, keepdim=True)
        acc = acc * alpha + torch.matmul(p, vf[:, j0:j1])
        m = m_new
    out = torch.where(den > 0, acc / den.clamp_min(1e-30), torch.zeros_like(acc))
    return out.to(query.dtype)


def sparse_attention(query, key, value, pattern_mask, scale: float | None = None):
    """Attention restricted to pattern_mask [Lq, Lk] (True = attended); rows without any attended
    key give zeros."""
    _check3(query, key, value)
    if tuple(pattern_mask.shape) != (query.shape[1], key.shape[1]):
        raise ValueError(f"pattern mask shape {tuple(pattern_mask.shape)} does not match "
                         f"[{query.shape[1]}, {key.shape[1]}]")
    scale = scale if scale is not None else query.shape[-1] ** -0.5
    return _scores_attention(query, key, value, scale, AttentionMask.boolean(pattern_mask[None]))


def attention_with_alibi(query, key, value, slopes, scale: float | None = None, causal: bool = False):
    _check3(query, key, value)
    scale = scale if scale is not None else query.shape[-1] ** -0.5
    Lq, Lk = query.shape[1], key.shape[1]
    pos = (torch.arange(Lq, device=query.device)[:, None] - torch.arange(Lk, device=query.device)[None, :]).abs()
    slope = torch.as_tensor(slopes, device=query.device).reshape(-1)[0]
    bias = (-slope * pos.to(slope.dtype if slope.is_floating_point() else torch.float32))[None]
    s = torch.matmul(query, key.transpose(-1, -2)) * scale + bias.to(query.dtype)
    if causal:
        tri = torch.ones(Lq, Lk, dtype=torch.bool, device=query.device).tril()
        s = s.masked_fill(~tri, float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, dim=-1), nan=0.0)
    return torch.matmul(p, value)


def rotary_embedding(x, freq_base: float = 10000.0):
    """RoPE on interleaved pairs of x [B, L, d] (d even)."""
    if x.dim() != 3:
        raise ValueError("x must be [batch, seq, d_model]")
    B, L, d = x.shape
    if d % 2:
        raise ValueError("model dimension must be even for rotary embeddings")
    i = torch.arange(d // 2, device=x.device, dtype=torch.float64)
    freqs = freq_base ** (-(2.0 * i) / d)
    theta = torch.arange(L, device=x.device, dtype=torch.float64)[:, None] * freqs[None, :]
    cos, sin = theta.cos().to(x.dtype), theta.sin().to(x.dtype)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * cos - x1 * sin
    out[..., 1::2] = x0 * sin + x1 * cos
    return out


def linear_attention(query, key, value, scale: float | None = None):
    """O(L) attention with the elu + 1 feature map: (q' (k'^T v)) / (q' . sum_k k')."""
    _check3(query, key, value)
    scale = scale if scale is not None else query.shape[-1] ** -0.5
    qp = F.elu(query) + 1.0
    kp = F.elu(key * scale) + 1.0
    kv = torch.matmul(kp.transpose(-1, -2), value)               # [B, d, dv]
    z = torch.matmul(qp, kp.sum(dim=1, keepdim=True).transpose(-1, -2))  # [B, Lq, 1]
    num = torch.matmul(qp, kv)
    return torch.where(z > 0, num / torch.where(z > 0, z, torch.ones_like(z)), torch.zeros_like(num))


def relative_position_attention(query, key, value, rel_emb, scale: float | None = None):
    _check3(query, key, value)
    Lq, Lk, d = query.shape[1], key.shape[1], query.shape[2]
    n = 2 * max(Lq, Lk) - 1
    if tuple(rel_emb.shape) != (n, d):
        raise ValueError(f"relative embedding shape should be [{n}, {d}], got {tuple(rel_emb.shape)}")
    scale = scale if scale is not None else d ** -0.5
    idx = (Lk - 1) + torch.arange(Lq, device=query.device)[:, None] - torch.arange(Lk, device=query.device)[None, :]
    content = torch.matmul(query, key.transpose(-1, -2))
    pos_all = torch.matmul(query, rel_emb.t())                    # [B, Lq, n]
    pos = torch.gather(pos_all, 2, idx[None].expand(query.shape[0], Lq, Lk))
    p = torch.softmax((content + pos) * scale, dim=-1)
    return torch.matmul(p, value)


def attention_with_rpe(query, key, value, rel_emb, scale: float | None = None, use_xpos: bool = False):
    if not use_xpos:
        return relative_position_attention(query, key, value, rel_emb, scale)
    _check3(query, key, value)
    d = query.shape[2]
    jf = torch.arange(d, device=query.device, dtype=torch.float64) / d

    def xpos(t):
        p = torch.arange(1, t.shape[1] + 1, device=t.device, dtype=torch.float64)[:, None]
        return t * (p ** (-jf[None, :])).to(t.dtype)

    return scaled_dot_product_attention(xpos(query), xpos(key), value, None, scale)


def _project(x, w):
    from ..ops import functional as OF

    return OF.linear(x, w)


def multi_head_attention(query, key, value, wq, wk, wv, wo, mask: AttentionMask | None, config: AttentionConfig):
    """Projections x @ W ([d_model, d_model] weights), config.num_heads heads of config.head_dim,
    attention (causal from the config or the mask), output projection."""
    _check3(query, key, value)
    B, Lq, d = query.shape
    H, hd = config.num_heads, config.head_dim
    if H * hd != d:
        raise ValueError(f"num_heads x head_dim = {H * hd} does not match d_model {d}")
    for w in (wq, wk, wv, wo):
        if tuple(w.shape) != (d, d):
            raise ValueError("weight matrices must be [d_model, d_model]")
    scale = config.scale if config.scale is not None else hd ** -0.5
    q = _project(query, wq).view(B, Lq, H, hd)
    k = _project(key, wk).view(B, key.shape[1], H, hd)
    v = _project(value, wv).view(B, value.shape[1], H, hd)
    causal = config.causal or (mask is not None and mask.kind == "causal")
    if mask is None or mask.kind == "causal":
        o = _heads_attention(q, k, v, causal, scale)
    else:
        o = _scores_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale,
                              AttentionMask(mask.kind, mask.tensor[:, None]), causal=config.causal)
        o = o.transpose(1, 2)
    if config.dropout_prob > 0 and torch.is_grad_enabled():
        o = F.dropout(o, config.dropout_prob)
    return _project(o.reshape(B, Lq, d), wo)


def grouped_query_attention(query, key, value, wq, wk, wv, wo, mask: AttentionMask | None, num_heads: int,
                            num_kv_heads: int, scale: float | None = None):
    """num_heads query heads share num_kv_heads key / value heads (wk / wv: [d_model, kv_dim])."""
    _check3(query, key, value)
    if num_heads % num_kv_heads:
        raise ValueError(f"number of heads ({num_heads}) must be divisible by number of key-value heads "
                         f"({num_kv_heads})")
    B, Lq, d = query.shape
    hd = d // num_heads
    kv_dim = num_kv_heads * hd
    if tuple(wq.shape) != (d, d) or tuple(wk.shape) != (d, kv_dim) or tuple(wv.shape) != (d, kv_dim) \
            or tuple(wo.shape) != (d, d):
        raise ValueError("weight matrices have incorrect dimensions")
    scale = scale if scale is not None else hd ** -0.5
    g = num_heads // num_kv_heads
    q = _project(query, wq).view(B, Lq, num_heads, hd)
    k = _project(key, wk).view(B, key.shape[1], num_kv_heads, hd).repeat_interleave(g, dim=2)
    v = _project(value, wv).view(B, value.shape[1], num_kv_heads, hd).repeat_interleave(g, dim=2)
    if mask is None or mask.kind == "causal":
        o = _heads_attention(q, k, v, mask is not None, scale)
    else:
        o = _scores_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale,
                              AttentionMask(mask.kind, mask.tensor[:, None])).transpose(1, 2)
    return _project(o.reshape(B, Lq, d), wo)
