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


class SparseTensor:
    """N-dimensional sparse tensor: sorted unique flat (row-major) indices
    with their values over a dense shape. Backed by torch COO tensors for
    products with dense operands, so `matmul` is differentiable with respect
    to the dense side and the values.

    Reference parity: scirs2-autograd/src/sparse/sparse_tensor.rs:17-260
    (new / zeros / from_dense / flat<->coords / to_dense / accumulate /
    reshape / slice_first_dim / to_sparse_grad)."""

    def __init__(self, shape, indices, values):
        self.shape = tuple(int(s) for s in shape)
        self.total = 1
        for s in self.shape:
            self.total *= s
        g = SparseGrad(indices, values, self.total)
        self.indices, self.values = g.indices, g.values

    @classmethod
    def zeros(cls, shape) -> "SparseTensor":
        return cls(shape, [], [])

    @classmethod
    def from_dense(cls, dense: torch.Tensor, threshold: float = 0.0) -> "SparseTensor":
        g = SparseGrad.from_dense(dense, threshold)
        return cls(dense.shape, g.indices, g.values)

    def total_size(self) -> int:
        return self.total

    def nnz(self) -> int:
        return int(self.indices.numel())

    def flat_to_coords(self, flat: int) -> list[int]:
        out = []
        for s in reversed(self.shape):
            out.append(flat % s)
            flat //= s
        return out[::-1]

    def coords_to_flat(self, coords) -> int:
        if len(coords) != len(self.shape) or any(not 0 <= c < s for c, s in zip(coords, self.shape)):
            raise ValueError(f"coordinates {coords} outside shape {self.shape}")
        f = 0
        for c, s in zip(coords, self.shape):
            f = f * s + int(c)
        return f

    def coords(self) -> torch.Tensor:
        """[ndim, nnz] coordinate matrix."""
        out, rem = [], self.indices.clone()
        for s in reversed(self.shape):
            out.append(rem % s)
            rem = rem // s
        return torch.stack(out[::-1]) if out else rem.reshape(0, 0)

    def to_dense(self) -> torch.Tensor:
        d = torch.zeros(self.total, dtype=self.values.dtype, device=self.values.device)
        d[self.indices] = self.values
        return d.reshape(self.shape)

    def to_torch(self) -> torch.Tensor:
        return torch.sparse_coo_tensor(self.coords(), self.values, self.shape).coalesce()

    def to_sparse_grad(self) -> SparseGrad:
        return SparseGrad(self.indices.clone(), self.values.clone(), self.total)

    def accumulate(self, other: "SparseTensor"):
        if other.shape != self.shape:
            raise ValueError(f"shape mismatch {self.shape} vs {other.shape}")
        g = SparseGrad(torch.cat([self.indices, other.indices]), torch.cat([self.values, other.values]), self.total)
        self.indices, self.values = g.indices, g.values

    def reshape(self, shape) -> "SparseTensor":
        t = SparseTensor.zeros(shape)
        if t.total != self.total:
            raise ValueError(f"cannot reshape {self.shape} to {tuple(shape)}")
        t.indices, t.values = self.indices.clone(), self.values.clone()
        return t

    def slice_first_dim(self, start: int, end: int) -> "SparseTensor":
        if not 0 <= start <= end <= self.shape[0]:
            raise ValueError("slice outside the first dimension")
        inner = self.total // self.shape[0] if self.shape[0] else 0
        keep = (self.indices >= start * inner) & (self.indices < end * inner)
        t = SparseTensor.zeros((end - start,) + self.shape[1:])
        t.indices, t.values = self.indices[keep] - start * inner, self.values[keep]
        return t

    def matmul(self, dense: torch.Tensor) -> torch.Tensor:
        """(sparse [m, k]) @ (dense [k, n]) -> dense [m, n]."""
        if len(self.shape) != 2:
            raise ValueError("matmul needs a 2-D sparse operand")
        return torch.sparse.mm(self.to_torch().to(dense.dtype), dense)


class SparseGradAccumulator:
    """Per-parameter gradient accumulation over steps, keeping sparse
    gradients sparse (reference: sparse_tensor.rs:290-380)."""

    def __init__(self):
        self.grads: dict[str, GradientRepr] = {}
        self.steps = 0

    def accumulate_sparse(self, name: str, grad: SparseGrad):
        if name in self.grads:
            self.grads[name].accumulate(GradientRepr(grad))
        else:
            self.grads[name] = GradientRepr(SparseGrad(grad.indices.clone(), grad.values.clone(), grad.shape))

    def accumulate_dense(self, name: str, grad: torch.Tensor):
        if name in self.grads:
            self.grads[name].accumulate(GradientRepr(grad.reshape(-1)))
        else:
            self.grads[name] = GradientRepr(grad.reshape(-1).clone())

    def step(self):
        self.steps += 1

    def num_steps(self) -> int:
        return self.steps

    def averaged_grad(self, name: str) -> torch.Tensor | None:
        if name not in self.grads:
            return None
        return self.grads[name].to_dense() / max(1, self.steps)

    def raw_grad(self, name: str):
        return self.grads.get(name)

    def param_names(self) -> list[str]:
        return sorted(self.grads)

    def clear(self):
        self.grads.clear()
        self.steps = 0


def embedding_backward(ids: torch.Tensor, grad_out: torch.Tensor, num_embeddings: int) -> SparseTensor:
    """Gradient of an embedding lookup as a sparse [num_embeddings, dim]
    tensor holding only the rows that were looked up (duplicates summed)."""
    dim = grad_out.shape[-1]
    ids = ids.reshape(-1).long()
    g = grad_out.reshape(-1, dim)
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= num_embeddings):
        raise ValueError("embedding id out of range")
    flat = (ids[:, None] * dim + torch.arange(dim, device=ids.device)[None, :]).reshape(-1)
    return SparseTensor((num_embeddings, dim), flat, g.reshape(-1).float())
