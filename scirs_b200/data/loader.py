"""Datasets and a GPU-feeding data loader.

`DataLoader` gathers batches on the host with the native prefetcher
(scirs_b200/csrc/dataloader.cpp: worker threads, seeded shuffle, ring of
pinned staging slots) and copies them to the device on a dedicated CUDA
stream, one batch ahead: the gather of batch i+2 and the host->device copy
of batch i+1 overlap the training step on batch i. Optional transforms run
on the device batch.

`DataLoader.stats()` reports batches / samples delivered, the host time spent
waiting for the prefetcher and the resulting throughput. `BatchSizeOptimizer`
times a training step (CUDA events on a device) over a range of batch sizes
and picks the fastest one that fits a memory budget; `MemoryAwareDataLoader`
derives its batch size from the free device (or host) memory.

Reference parity: scirs2-neural/src/data/dataset.rs (Dataset,
InMemoryDataset), dataloader.rs:18-168 (DataLoader: batch_size, shuffle,
drop_last), transforms.rs / augmentation.rs (normalise, flips, noise, crops),
training/optimized_dataloader.rs:33-1066 (LoadingStats, BatchSizeOptimizer,
MemoryAwareDataLoader with an adaptive batch size).
"""
from __future__ import annotations

import dataclasses
import time
from typing import Callable

import torch

from .. import _ext


class Dataset:
    def __len__(self) -> int:
        raise NotImplementedError

    def get(self, i: int):
        raise NotImplementedError


class InMemoryDataset(Dataset):
    """Arrays sharing their first (sample) dimension."""

    def __init__(self, *arrays):
        self.arrays = [torch.as_tensor(a).contiguous() for a in arrays]
        n = self.arrays[0].shape[0]
        assert all(a.shape[0] == n for a in self.arrays), "arrays must share their first dimension"

    def __len__(self) -> int:
        return self.arrays[0].shape[0]

    def get(self, i: int):
        return tuple(a[i] for a in self.arrays)

    def train_test_split(self, test_fraction: float = 0.2, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(len(self), generator=g)
        k = int(round(len(self) * (1 - test_fraction)))
        return (InMemoryDataset(*(a[perm[:k]] for a in self.arrays)),
                InMemoryDataset(*(a[perm[k:]] for a in self.arrays)))


class DataLoader:
    def __init__(self, dataset: InMemoryDataset, batch_size: int, shuffle: bool = True, drop_last: bool = False,
                 num_workers: int = 2, seed: int = 0, device=None, transforms=None, prefetch_slots: int = 3):
        self.dataset = dataset
        self.batch_size = batch_size
        self.device = torch.device(device) if device is not None else None
        self.transforms = list(transforms or [])
        pin = self.device is not None and self.device.type == "cuda"
        self.pf = _ext.data().BatchPrefetcher(dataset.arrays, batch_size, max(2, prefetch_slots), max(1, num_workers),
                                              shuffle, seed, drop_last, pin)
        self.epoch = 0
        self.stream = torch.cuda.Stream(self.device) if pin else None
        self._stats = LoadingStats()

    def stats(self) -> "LoadingStats":
        return dataclasses.replace(self._stats)

    def reset_stats(self) -> None:
        self._stats = LoadingStats()

    def _next(self):
        t0 = time.perf_counter()
        r = self.pf.next()
        self._stats.wait_time_s += time.perf_counter() - t0
        if r[0] >= 0:
            self._stats.batches_loaded += 1
            self._stats.samples_loaded += int(r[1])
        return r

    def __len__(self) -> int:
        return self.pf.num_batches()

    def _to_device(self, host):
        """Copy a held batch on the copy stream; returns (tensors, event)."""
        if self.stream is None:
            return [h.clone() for h in host], None
        with torch.cuda.stream(self.stream):
            dev = [h.to(self.device, non_blocking=True) for h in host]
            ev = torch.cuda.Event()
            ev.record(self.stream)
        return dev, ev

    def __iter__(self):
        self.pf.start_epoch(self.epoch)
        self.epoch += 1
        self._stats.epoch_start = time.perf_counter()
        slot, rows, host = self._next()
        pending = None
        if slot >= 0:
            pending = (slot, *self._to_device(host))
        while pending is not None:
            slot, dev, ev = pending
            nslot, _, nhost = self._next()
            nxt = (nslot, *self._to_device(nhost)) if nslot >= 0 else None
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
                for t in dev:
                    t.record_stream(torch.cuda.current_stream(self.device))
                ev.synchronize()  # the pinned slot may be refilled once its copy finished
            self.pf.release(slot)
            batch = tuple(dev)
            for tf in self.transforms:
                batch = tf(batch)
            yield batch if len(batch) > 1 else batch[0]
            pending = nxt
        self._stats.elapsed_s += time.perf_counter() - self._stats.epoch_start


@dataclasses.dataclass
class LoadingStats:
    batches_loaded: int = 0
    samples_loaded: int = 0
    wait_time_s: float = 0.0  # host time spent waiting for the prefetcher
    elapsed_s: float = 0.0  # wall time of finished epochs
    epoch_start: float = 0.0

    @property
    def avg_wait_ms(self) -> float:
        return 1e3 * self.wait_time_s / max(1, self.batches_loaded)

    @property
    def samples_per_second(self) -> float:
        return self.samples_loaded / self.elapsed_s if self.elapsed_s > 0 else 0.0


@dataclasses.dataclass
class BatchSizeOptimizationResult:
    recommended_batch_size: int
    throughput_results: list  # [(batch size, samples / s)]
    memory_results: list  # [(batch size, bytes)]
    memory_limited: bool


class BatchSizeOptimizer:
    """Tries batch sizes min, 2*min, ... up to max. For each it runs `warmup` then `timing` batches
    through `step_fn(batch)` (or only loads them), timing with CUDA events on a device, and records
    the peak device memory of the step (host batch bytes without a device). The fastest size whose
    memory stays within `max_memory` (0: no limit) is recommended; the search stops at the first
    size over the limit."""

    def __init__(self, min_batch_size: int = 8, max_batch_size: int = 512, warmup_batches: int = 2,
                 timing_batches: int = 5, max_memory: int = 0):
        self.min, self.max = min_batch_size, max_batch_size
        self.warmup, self.timing, self.max_memory = warmup_batches, timing_batches, max_memory

    def with_range(self, lo: int, hi: int) -> "BatchSizeOptimizer":
        self.min, self.max = lo, hi
        return self

    def with_max_memory(self, max_memory: int) -> "BatchSizeOptimizer":
        self.max_memory = max_memory
        return self

    def find_optimal(self, dataset: "InMemoryDataset", step_fn: Callable | None = None,
                     device=None) -> BatchSizeOptimizationResult:
        dev = torch.device(device) if device is not None else None
        cuda = dev is not None and dev.type == "cuda"
        thr, mem = [], []
        best, best_thr, limited = self.min, -1.0, False
        bs = self.min
        while bs <= self.max and bs <= len(dataset):
            loader = DataLoader(dataset, bs, shuffle=False, drop_last=True, device=dev)
            it = iter(loader)
            batches = []
            for _ in range(self.warmup + self.timing):
                try:
                    batches.append(next(it))
                except StopIteration:
                    break
            if len(batches) <= self.warmup:
                break
            for b in batches[: self.warmup]:
                if step_fn is not None:
                    step_fn(b)
            timed = batches[self.warmup:]
            if cuda:
                torch.cuda.synchronize(dev)
                torch.cuda.reset_peak_memory_stats(dev)
                base = torch.cuda.memory_allocated(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            t0 = time.perf_counter()
            for b in timed:
                if step_fn is not None:
                    step_fn(b)
            if cuda:
                e1.record()
                torch.cuda.synchronize(dev)
                secs = e0.elapsed_time(e1) / 1e3
                used = torch.cuda.max_memory_allocated(dev) - base + sum(
                    t.numel() * t.element_size() for t in (timed[0] if isinstance(timed[0], tuple) else (timed[0],)))
            else:
                secs = time.perf_counter() - t0
                used = sum(t.numel() * t.element_size() for t in (timed[0] if isinstance(timed[0], tuple)
                                                                    else (timed[0],)))
            sps = len(timed) * bs / max(secs, 1e-9)
            thr.append((bs, sps))
            mem.append((bs, int(used)))
            if self.max_memory and used > self.max_memory:
                limited = True
                break
            if sps > best_thr:
                best, best_thr = bs, sps
            bs *= 2
        return BatchSizeOptimizationResult(best, thr, mem, limited)


class MemoryAwareDataLoader:
    """A DataLoader whose batch size is floor(budget / (bytes per sample * overhead)), clamped to
    [min, max] and rounded down to a multiple of `multiple` (8 keeps GEMM shapes tensor-core
    aligned). The budget is `memory_fraction` of the free device memory (of the host's available
    memory without a device) unless given in bytes."""

    def __init__(self, dataset: "InMemoryDataset", memory_budget: int | None = None, memory_fraction: float = 0.1,
                 overhead_factor: float = 4.0, min_batch_size: int = 1, max_batch_size: int = 4096,
                 multiple: int = 8, device=None, **loader_kw):
        self.dataset, self.budget, self.fraction = dataset, memory_budget, memory_fraction
        self.overhead, self.lo, self.hi, self.multiple = overhead_factor, min_batch_size, max_batch_size, multiple
        self.device, self.loader_kw = device, loader_kw
        self.sample_bytes = sum(a[0].numel() * a.element_size() for a in dataset.arrays)
        self._loader: DataLoader | None = None
        self.refresh_batch_size()

    def _budget(self) -> int:
        if self.budget is not None:
            return int(self.budget)
        dev = torch.device(self.device) if self.device is not None else None
        if dev is not None and dev.type == "cuda":
            return int(torch.cuda.mem_get_info(dev)[0] * self.fraction)
        import psutil

        return int(psutil.virtual_memory().available * self.fraction)

    def refresh_batch_size(self) -> int:
        bs = int(self._budget() // max(1.0, self.sample_bytes * self.overhead))
        bs = max(self.lo, min(self.hi, bs, len(self.dataset)))
        if bs >= self.multiple:
            bs -= bs % self.multiple
        self.batch_size = max(self.lo, bs)
        self._loader = DataLoader(self.dataset, self.batch_size, device=self.device, **self.loader_kw)
        return self.batch_size

    def adaptive_batch_size(self) -> int:
        return self.batch_size

    def __len__(self) -> int:
        return len(self._loader)

    def stats(self) -> LoadingStats:
        return self._loader.stats()

    def __iter__(self):
        return iter(self._loader)


# ---------------------------------------------------------------- transforms
class Normalize:
    """(x - mean) / std on the first tensor of the batch (per channel dim 1)."""

    def __init__(self, mean, std):
        self.mean, self.std = torch.as_tensor(mean), torch.as_tensor(std)

    def __call__(self, batch):
        x = batch[0].float()
        shape = [1, -1] + [1] * (x.dim() - 2)
        x = (x - self.mean.to(x.device).view(shape)) / self.std.to(x.device).view(shape)
        return (x,) + tuple(batch[1:])


class RandomHorizontalFlip:
    def __init__(self, p: float = 0.5, seed: int = 0):
        self.p = p
        self.g = torch.Generator().manual_seed(seed)

    def __call__(self, batch):
        x = batch[0]
        flip = (torch.rand(x.shape[0], generator=self.g) < self.p).to(x.device)
        x = torch.where(flip.view(-1, *([1] * (x.dim() - 1))), x.flip(-1), x)
        return (x,) + tuple(batch[1:])


class GaussianNoise:
    def __init__(self, std: float = 0.01, seed: int = 0):
        self.std = std
        self.g = torch.Generator().manual_seed(seed)

    def __call__(self, batch):
        x = batch[0]
        n = torch.randn(x.shape, generator=self.g).to(x.device, x.dtype) * self.std
        return (x + n,) + tuple(batch[1:])


class RandomCrop:
    """Pad by `padding` then crop back to the original size at a random offset
    (one offset per batch)."""

    def __init__(self, padding: int = 4, seed: int = 0):
        self.padding = padding
        self.g = torch.Generator().manual_seed(seed)

    def __call__(self, batch):
        x = batch[0]
        p = self.padding
        H, W = x.shape[-2:]
        xp = torch.nn.functional.pad(x, (p, p, p, p))
        i, j = (int(v) for v in torch.randint(0, 2 * p + 1, (2,), generator=self.g))
        return (xp[..., i : i + H, j : j + W],) + tuple(batch[1:])
