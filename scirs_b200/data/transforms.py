"""Feature transforms, dataset wrappers and split utilities.

  StandardScaler(fit_per_sample)   (x - mean) / std, statistics over samples (per feature), or per
                                   sample over its features; 1-D data uses one global mean / std;
                                   a zero std divides by 1
  MinMaxScaler(feature_range)      x -> lo + (x - min) / (max - min) * (hi - lo), per feature
  OneHotEncoder(n_classes)         integer labels [N] or [N, 1] -> [N, n_classes]
  ComposeTransform(transforms)     applies them in order
  CSVDataset / TransformedDataset / SubsetDataset   dataset wrappers
  train_val_split(x, y, val_size, shuffle, seed)    val count = round(N * val_size), both non-empty
  KFold(n_splits, shuffle, random_state).split(n)   folds of size n // k, the first n % k one larger
  create_batches(x, y, batch_size, shuffle, seed)   list of (x, y) batches

Reference parity: scirs2-neural/src/data/transforms.rs:10-430,
data/dataset.rs:13-300, data/utils.rs:18-230.
"""
from __future__ import annotations

import csv

import torch

from .loader import Dataset


class Transform:
    def fit(self, x):
        return self

    def transform(self, x):
        raise NotImplementedError

    def fit_transform(self, x):
        return self.fit(x).transform(x)

    def __call__(self, x):
        return self.transform(x)


class StandardScaler(Transform):
    def __init__(self, fit_per_sample: bool = False):
        self.fit_per_sample, self.mean, self.std = fit_per_sample, None, None

    def fit(self, x):
        x = torch.as_tensor(x, dtype=torch.float64)
        if x.dim() < 2:
            self.mean, self.std = x.mean().reshape(1), x.std(unbiased=False).reshape(1)
        elif self.fit_per_sample:
            self.mean, self.std = x.mean(1), x.std(1, unbiased=False)
        else:
            self.mean, self.std = x.mean(0), x.std(0, unbiased=False)
        return self

    def transform(self, x):
        if self.mean is None:
            raise RuntimeError("StandardScaler has not been fitted")
        x = torch.as_tensor(x, dtype=torch.float64)
        std = torch.where(self.std == 0, torch.ones_like(self.std), self.std)
        if x.dim() >= 2 and self.fit_per_sample:
            return (x - self.mean[:, None]) / std[:, None]
        return (x - self.mean) / std

    def inverse_transform(self, y):
        std = torch.where(self.std == 0, torch.ones_like(self.std), self.std)
        if y.dim() >= 2 and self.fit_per_sample:
            return y * std[:, None] + self.mean[:, None]
        return y * std + self.mean


class MinMaxScaler(Transform):
    def __init__(self, feature_range=(0.0, 1.0)):
        lo, hi = feature_range
        if not lo < hi:
            raise ValueError("feature_range must be increasing")
        self.lo, self.hi, self.min, self.max = float(lo), float(hi), None, None

    def fit(self, x):
        x = torch.as_tensor(x, dtype=torch.float64)
        self.min, self.max = (x.min(0).values, x.max(0).values) if x.dim() >= 2 else (x.min(), x.max())
        return self

    def transform(self, x):
        if self.min is None:
            raise RuntimeError("MinMaxScaler has not been fitted")
        x = torch.as_tensor(x, dtype=torch.float64)
        rng = self.max - self.min
        rng = torch.where(rng == 0, torch.ones_like(rng), rng)
        return self.lo + (x - self.min) / rng * (self.hi - self.lo)


class OneHotEncoder(Transform):
    def __init__(self, n_classes: int):
        if n_classes < 1:
            raise ValueError("n_classes must be positive")
        self.n_classes = n_classes

    def transform(self, y):
        y = torch.as_tensor(y).reshape(-1).long()
        if (y < 0).any() or (y >= self.n_classes).any():
            raise ValueError(f"labels must be in [0, {self.n_classes})")
        return torch.nn.functional.one_hot(y, self.n_classes).to(torch.float64)


class ComposeTransform(Transform):
    def __init__(self, transforms):
        self.transforms = list(transforms)

    def fit(self, x):
        for t in self.transforms:
            x = t.fit_transform(x)
        return self

    def transform(self, x):
        for t in self.transforms:
            x = t.transform(x)
        return x


class CSVDataset(Dataset):
    """Rows of a CSV file; `label_cols` (indices) become the targets, the rest the features."""

    def __init__(self, path: str, label_cols=(-1,), has_header: bool = True, delimiter: str = ","):
        with open(path, newline="") as f:
            rows = list(csv.reader(f, delimiter=delimiter))
        if has_header:
            self.header, rows = rows[0], rows[1:]
        else:
            self.header = None
        data = torch.tensor([[float(v) for v in r] for r in rows if r], dtype=torch.float64)
        ncol = data.shape[1]
        lab = sorted({c % ncol for c in label_cols})
        feat = [c for c in range(ncol) if c not in lab]
        self.features, self.labels = data[:, feat], data[:, lab]

    def __len__(self):
        return self.features.shape[0]

    def get(self, i):
        return self.features[i], self.labels[i]


class TransformedDataset(Dataset):
    def __init__(self, dataset: Dataset, feature_transform=None, label_transform=None):
        self.dataset, self.ft, self.lt = dataset, feature_transform, label_transform

    def __len__(self):
        return len(self.dataset)

    def get(self, i):
        x, y = self.dataset.get(i)[:2]
        x = self.ft(x[None])[0] if self.ft is not None else x
        y = self.lt(y[None])[0] if self.lt is not None else y
        return x, y


class SubsetDataset(Dataset):
    def __init__(self, dataset: Dataset, indices):
        self.dataset, self.indices = dataset, [int(i) for i in indices]
        if any(i < 0 or i >= len(dataset) for i in self.indices):
            raise IndexError("subset index out of range")

    def __len__(self):
        return len(self.indices)

    def get(self, i):
        return self.dataset.get(self.indices[i])


def train_val_split(x, y, val_size: float, shuffle: bool = True, seed: int = 0):
    if not 0.0 < val_size < 1.0:
        raise ValueError("Validation size must be between 0 and 1")
    n = x.shape[0]
    if n != y.shape[0]:
        raise ValueError(f"X and y have different number of samples: {n} vs {y.shape[0]}")
    n_val = int(round(n * val_size))
    if n_val == 0 or n_val == n:
        raise ValueError("Split would result in empty training or validation set")
    idx = torch.randperm(n, generator=torch.Generator().manual_seed(seed)) if shuffle else torch.arange(n)
    tr, va = idx[: n - n_val], idx[n - n_val:]
    return x[tr], x[va], y[tr], y[va]


class KFold:
    def __init__(self, n_splits: int = 5, shuffle: bool = False, random_state: int | None = None):
        self.n_splits, self.shuffle, self.random_state = n_splits, shuffle, random_state

    def split(self, n_samples: int):
        if self.n_splits < 2:
            raise ValueError("n_splits must be >= 2")
        if self.n_splits > n_samples:
            raise ValueError("n_splits must be <= n_samples")
        if self.shuffle:
            g = torch.Generator()
            g.manual_seed(self.random_state if self.random_state is not None else torch.seed())
            idx = torch.randperm(n_samples, generator=g).tolist()
        else:
            idx = list(range(n_samples))
        sizes = [n_samples // self.n_splits + (1 if i < n_samples % self.n_splits else 0)
                 for i in range(self.n_splits)]
        out, cur = [], 0
        for s in sizes:
            test = idx[cur:cur + s]
            out.append((idx[:cur] + idx[cur + s:], test))
            cur += s
        return out


def create_batches(x, y, batch_size: int, shuffle: bool = False, seed: int = 0):
    if batch_size < 1:
        raise ValueError("batch_size must be positive")
    n = x.shape[0]
    idx = torch.randperm(n, generator=torch.Generator().manual_seed(seed)) if shuffle else torch.arange(n)
    return [(x[idx[i:i + batch_size]], y[idx[i:i + batch_size]]) for i in range(0, n, batch_size)]
