"""Sparse gradients: (indices, values) over a flat dense shape, for
embedding-style updates and top-k gradient exchange.

Reference parity: scirs2-autograd/src/sparse/sparse_tensor.rs:41-340
(SparseGrad: from_dense with a threshold, to_dense, nnz / sparsity,
sparsify, accumulate / merge, add_to_dense, scale, clip, norms;
GradientRepr dense-or-sparse with accumulation).
"""
from __future__ import annotations

import torch


class SparseGrad:
    def __init__(self, indices, values, shape: int):
        idx = torch.as_tensor(indices, dtype=torch.long)
        val = torch.as_tensor(values, dtype=torch.float32, device=idx.device)
        if idx.shape != val.shape:
            raise ValueError("indices and values must have the same length")
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= shape):
            raise ValueError("index out of range")
        self.shape = int(shape)
        self._coalesce(idx, val)

    def _coalesce(self, idx, val):
        if idx.numel():
            uniq, inv = torch.unique(idx, sorted=True, return_inverse=True)
            acc = torch.zeros(uniq.numel(), dtype=val.dtype, device=val.device).index_add_(0, inv, val)
            idx, val = uniq, acc
        self.indices, self.values = idx, val

    @classmethod
    def zeros(cls, shape: int) -> "SparseGrad":
        return cls([], [], shape)

    @classmethod
    def from_dense(cls, dense: torch.Tensor, threshold: float = 0.0) -> "SparseGrad":
        d = dense.reshape(-1)
        idx = torch.nonzero(d.abs() > threshold).reshape(-1)
        return cls(idx, d[idx].float(), d.numel())

    def to_dense(self) -> torch.Tensor:
        out = torch.zeros(self.shape, dtype=self.values.dtype, device=self.values.device)
        out[self.indices] = self.values
        return out

    def nnz(self) -> int:
        return int(self.indices.numel())

    def sparsity(self) -> float:
        return 1.0 - self.nnz() / self.shape if self.shape else 1.0

    def sparsify(self, threshold: float):
        keep = self.values.abs() > threshold
        self.indices, self.values = self.indices[keep], self.values[keep]

    def accumulate(self, other: "SparseGrad"):
        if other.shape != self.shape:
            raise ValueError("shape mismatch")
        self._coalesce(torch.cat([self.indices, other.indices.to(self.indices.device)]),
                       torch.cat([self.values, other.values.to(self.values.device)]))

    @staticmethod
    def merge(a: "SparseGrad", b: "SparseGrad") -> "SparseGrad":
        out = SparseGrad(a.indices.clone(), a.values.clone(), a.shape)
        out.accumulate(b)
        return out

    def add_to_dense(self, dense: torch.Tensor):
        if dense.numel() != self.shape:
            raise ValueError("shape mismatch")
        dense.view(-1).index_add_(0, self.indices.to(dense.device), self.values.to(dense.device, dense.dtype))

    def scale(self, factor: float):
        self.values = self.values * factor

    def scaled(self, factor: float) -> "SparseGrad":
        return SparseGrad(self.indices.clone(), self.values * factor, self.shape)

    def clip(self, max_abs: float):
        self.values = self.values.clamp(-max_abs, max_abs)

    def l2_norm(self) -> float:
        return float(self.values.norm())

    def l1_norm(self) -> float:
        return float(self.values.abs().sum())


class GradientRepr:
    """A gradient held dense or sparse; accumulation keeps it sparse while
    both sides are sparse, otherwise densifies."""

    def __init__(self, value):
        self.value = value

    def is_sparse(self) -> bool:
        return isinstance(self.value, SparseGrad)

    def shape(self) -> int:
        return self.value.shape if self.is_sparse() else self.value.numel()

    def to_dense(self) -> torch.Tensor:
        return self.value.to_dense() if self.is_sparse() else self.value.reshape(-1)

    def to_sparse(self, threshold: float = 0.0) -> SparseGrad:
        return self.value if self.is_sparse() else SparseGrad.from_dense(self.value, threshold)

    def accumulate(self, other: "GradientRepr"):
        if self.is_sparse() and other.is_sparse():
            self.value.accumulate(other.value)
        else:
            d = self.to_dense().clone()
            if other.is_sparse():
                other.value.add_to_dense(d)
            else:
                d += other.to_dense().to(d.device, d.dtype)
            self.value = d
