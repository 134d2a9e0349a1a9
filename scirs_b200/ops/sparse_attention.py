"""Sparse and windowed attention without dense masks.

An attention pattern is an element predicate over (query q, key k): the
union of the components given, intersected with the causal mask,

    allowed(q, k) = (not causal or k <= q) and (
                        q - wl <= k <= q + wr            sliding window
                     or q < ng or k < ng                 global tokens
                     or bitmap[q // 128, k // 128])      block-sparse layout

(with no component given, every pair is allowed). This covers Longformer
(window + global), BigBird (window + global + random blocks) and Sparse
Transformer (local + strided blocks) patterns.

`AttentionPattern.plan(Sq, Sk, head_dim, device)` turns it into the block
lists the tcgen05 kernels walk:

  forward   for every CTA of 256 queries, the 128-key blocks it must visit
  backward  for every 128-key tile, the query blocks (128 queries for
            head_dim 64, 64 for head_dim 128) that see any of its keys

A block is listed when the interval test says some pair inside it may be
allowed (a superset; the kernels mask element by element), so the work is
O(S x window) instead of O(S^2) and no S x S mask is ever built. Plans are
cached per (shape, pattern, device).

Reference parity: scirs2-neural/src/attention/sliding_window.rs:39-219
(symmetric window + global tokens) and attention/sparse/attention.rs:40-218
(block-sparse patterns); CPU loops over the dense score matrix there.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

_FWD_Q = 256  # queries per forward CTA
_KB = 128  # keys per block (forward) / key tile (backward)


@dataclass(frozen=True)
class AttentionPattern:
    causal: bool = False
    window_left: int | None = None  # wl; None: no window
    window_right: int | None = None  # wr; defaults to window_left (symmetric), 0 when causal
    num_global: int = 0
    bitmap: torch.Tensor | None = field(default=None, compare=False, hash=False)  # [ceil(Sq/128), ceil(Sk/128)]
    bitmap_key: str | None = None  # identifies the bitmap in the plan cache

    @property
    def wl(self) -> int:
        return -1 if self.window_left is None else int(self.window_left)

    @property
    def wr(self) -> int:
        if self.window_left is None:
            return -1
        if self.window_right is not None:
            return int(self.window_right)
        return 0 if self.causal else int(self.window_left)

    # ------------------------------------------------------------ predicate
    def _has_components(self) -> bool:
        return self.window_left is not None or self.num_global > 0 or self.bitmap is not None

    def allowed_dense(self, Sq: int, Sk: int, device=None) -> torch.Tensor:
        """The [Sq, Sk] boolean mask (reference / tests only; O(S^2))."""
        q = torch.arange(Sq, device=device)[:, None]
        k = torch.arange(Sk, device=device)[None, :]
        if self._has_components():
            m = torch.zeros(Sq, Sk, dtype=torch.bool, device=device)
            if self.window_left is not None:
                m |= (k >= q - self.wl) & (k <= q + self.wr)
            if self.num_global > 0:
                m |= (q < self.num_global) | (k < self.num_global)
            if self.bitmap is not None:
                m |= self.bitmap.to(device=device, dtype=torch.bool)[q // 128, k // 128]
        else:
            m = torch.ones(Sq, Sk, dtype=torch.bool, device=device)
        if self.causal:
            m &= k <= q
        return m

    def _block_maybe(self, qa, qb, ka, kb) -> torch.Tensor:
        """[nq, nk] bool: may a pair inside query block [qa, qb] x key block
        [ka, kb] be allowed (inclusive bounds, broadcast tensors)."""
        shape = torch.broadcast_shapes(qa.shape, ka.shape)
        if self._has_components():
            ok = torch.zeros(shape, dtype=torch.bool)
            if self.window_left is not None:
                ok |= (kb >= qa - self.wl) & (ka <= qb + self.wr)
            if self.num_global > 0:
                ok |= (qa < self.num_global) | (ka < self.num_global)
            if self.bitmap is not None:
                bm = self.bitmap.to(torch.bool).cpu()
                # any 128-block covered by the (q, k) ranges
                q0, q1 = qa // 128, qb // 128
                k0, k1 = ka // 128, kb // 128
                cum = torch.zeros(bm.shape[0] + 1, bm.shape[1] + 1, dtype=torch.int64)
                cum[1:, 1:] = bm.long().cumsum(0).cumsum(1)
                tot = cum[q1 + 1, k1 + 1] - cum[q0, k1 + 1] - cum[q1 + 1, k0] + cum[q0, k0]
                ok |= tot > 0
        else:
            ok = torch.ones(shape, dtype=torch.bool)
        if self.causal:
            ok &= ka <= qb
        return ok

    def _csr(self, ok: torch.Tensor, transpose: bool):
        m = ok.t() if transpose else ok
        counts = m.sum(1).to(torch.int32)
        ptr = torch.zeros(m.shape[0] + 1, dtype=torch.int32)
        ptr[1:] = counts.cumsum(0)
        idx = m.nonzero()[:, 1].to(torch.int32)  # row-major order: sorted per row
        return ptr, idx

    def plan(self, Sq: int, Sk: int, head_dim: int, device) -> "AttentionPlan":
        key = (Sq, Sk, head_dim, str(device), self.causal, self.window_left, self.window_right, self.num_global,
               self.bitmap_key if self.bitmap is not None else None)
        hit = _PLANS.get(key)
        if hit is not None:
            return hit
        # forward: CTAs of 256 queries x 128-key blocks
        nqc, nkb = (Sq + _FWD_Q - 1) // _FWD_Q, (Sk + _KB - 1) // _KB
        qa = (torch.arange(nqc) * _FWD_Q)[:, None]
        qb = torch.clamp(qa + _FWD_Q - 1, max=Sq - 1)
        ka = (torch.arange(nkb) * _KB)[None, :]
        kb = torch.clamp(ka + _KB - 1, max=Sk - 1)
        fptr, fidx = self._csr(self._block_maybe(qa, qb, ka, kb), False)
        # backward: 128-key tiles x query blocks of BQ
        BQ = 128 if head_dim == 64 else 64
        nqb = (Sq + BQ - 1) // BQ
        qa2 = (torch.arange(nqb) * BQ)[:, None]
        qb2 = torch.clamp(qa2 + BQ - 1, max=Sq - 1)
        bptr, bidx = self._csr(self._block_maybe(qa2, qb2, ka, kb), True)
        bmap = None
        if self.bitmap is not None:
            bm = self.bitmap.to(torch.uint8)
            if bm.shape != ((Sq + 127) // 128, (Sk + 127) // 128):
                raise ValueError(f"bitmap must be [{(Sq + 127) // 128}, {(Sk + 127) // 128}]")
            bmap = bm.contiguous().to(device)
        p = AttentionPlan(self, Sq, Sk, fptr.to(device), fidx.to(device), bptr.to(device), bidx.to(device), bmap,
                          visited_fwd=int(fidx.numel()), dense_fwd=nqc * nkb)
        _PLANS[key] = p
        return p


@dataclass
class AttentionPlan:
    pattern: AttentionPattern
    Sq: int
    Sk: int
    fwd_ptr: torch.Tensor
    fwd_idx: torch.Tensor
    bwd_ptr: torch.Tensor
    bwd_idx: torch.Tensor
    bmap: torch.Tensor | None
    visited_fwd: int = 0
    dense_fwd: int = 0

    def kernel_args(self, backward: bool = False) -> dict:
        p = self.pattern
        return {
            "blk_ptr": self.bwd_ptr if backward else self.fwd_ptr,
            "blk_idx": self.bwd_idx if backward else self.fwd_idx,
            "bmap": self.bmap,
            "wl": p.wl,
            "wr": p.wr,
            "ng": int(p.num_global),
        }

    @property
    def density(self) -> float:
        """Fraction of the dense forward key blocks the kernels visit."""
        return self.visited_fwd / max(1, self.dense_fwd)


_PLANS: dict = {}


def sliding_window(window: int, num_global: int = 0, causal: bool = False) -> AttentionPattern:
    """Token i attends to [i - window, i + window] (or [i - window, i] when
    causal) plus the first `num_global` tokens, which attend to everything."""
    return AttentionPattern(causal=causal, window_left=int(window), num_global=int(num_global))


def block_sparse(bitmap: torch.Tensor, causal: bool = False, key: str | None = None) -> AttentionPattern:
    """Block-sparse pattern over 128 x 128 blocks (bitmap [q blocks, k blocks])."""
    bm = bitmap.to(torch.bool).cpu()
    k = key or f"bm{tuple(bm.shape)}:{hash(bytes(bm.to(torch.uint8).numpy().tobytes()))}"
    return AttentionPattern(causal=causal, bitmap=bm, bitmap_key=k)


def strided_bitmap(nq: int, nk: int, local: int = 1, stride: int = 4, causal: bool = False) -> torch.Tensor:
    """Sparse-Transformer style block layout: the `local` nearest key blocks
    of every query block plus every `stride`-th key block."""
    qi = torch.arange(nq)[:, None]
    ki = torch.arange(nk)[None, :]
    m = ((qi - ki).abs() < local) | ((ki % stride) == (stride - 1))
    if causal:
        m &= ki <= qi
    return m


def reference_attention(q, k, v, pattern: AttentionPattern, scale: float):
    """fp32 attention with the dense mask of `pattern` (oracle for tests and
    the CPU path). q [B, Sq, H, D], k / v [B, Sk, H, D]."""
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    s = (qf @ kf.transpose(-1, -2)) * scale
    m = pattern.allowed_dense(q.shape[1], k.shape[1], device=q.device)
    s = s.masked_fill(~m, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse[..., None]).nan_to_num(0.0)
    o = (p @ vf).transpose(1, 2)
    return o, lse
