"""Datasets and a GPU-feeding data loader.

`DataLoader` gathers batches on the host with the native prefetcher
(scirs_b200/csrc/dataloader.cpp: worker threads, seeded shuffle, ring of
pinned staging slots) and copies them to the device on a dedicated CUDA
stream, one batch ahead: the gather of batch i+2 and the host->device copy
of batch i+1 overlap the training step on batch i. Optional transforms run
on the device batch.

Reference parity: scirs2-neural/src/data/dataset.rs (Dataset,
InMemoryDataset), dataloader.rs:18-168 (DataLoader: batch_size, shuffle,
drop_last), transforms.rs / augmentation.rs (normalise, flips, noise, crops).
"""
from __future__ import annotations

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
        slot, rows, host = self.pf.next()
        pending = None
        if slot >= 0:
            pending = (slot, *self._to_device(host))
        while pending is not None:
            slot, dev, ev = pending
            nslot, _, nhost = self.pf.next()
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
