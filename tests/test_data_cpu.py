"""Native batch prefetcher and DataLoader (host side)."""
import torch

from scirs_b200.data import DataLoader, InMemoryDataset, Normalize, RandomCrop, RandomHorizontalFlip


def test_loader_covers_every_sample_once_per_epoch():
    x = torch.arange(103 * 3, dtype=torch.float32).view(103, 3)
    y = torch.arange(103)
    dl = DataLoader(InMemoryDataset(x, y), batch_size=10, shuffle=True, num_workers=3, seed=5)
    assert len(dl) == 11
    seen = []
    for xb, yb in dl:
        assert torch.equal(xb, x[yb])  # rows gathered consistently across arrays
        seen += yb.tolist()
    assert sorted(seen) == list(range(103)) and seen != list(range(103))
    order2 = [int(v) for _, yb in dl for v in yb]
    assert order2 != seen and sorted(order2) == list(range(103))  # new order each epoch


def test_loader_sequential_drop_last_and_transforms():
    x = torch.arange(25, dtype=torch.float32).view(25, 1, 1, 1).repeat(1, 3, 4, 4)
    dl = DataLoader(InMemoryDataset(x), batch_size=8, shuffle=False, drop_last=True,
                    transforms=[Normalize([1.0, 1.0, 1.0], [2.0, 2.0, 2.0]), RandomHorizontalFlip(0.5),
                                RandomCrop(1)])
    batches = list(dl)
    assert len(batches) == 3 and all(b.shape == (8, 3, 4, 4) for b in batches)
    assert float(batches[0][1, 0, 1, 1]) == 0.0  # (1 - 1) / 2 at an interior pixel
    assert len(InMemoryDataset(x).train_test_split(0.2)[1]) == 5
