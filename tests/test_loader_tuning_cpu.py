"""Loader statistics, batch-size search and the memory-aware loader (host
paths; the device path times with CUDA events)."""
import time

import torch

from scirs_b200.data.loader import BatchSizeOptimizer, DataLoader, InMemoryDataset, MemoryAwareDataLoader


def _ds(n=512, d=16):
    g = torch.Generator().manual_seed(0)
    return InMemoryDataset(torch.randn(n, d, generator=g), torch.randint(0, 3, (n,), generator=g))


def test_loading_stats_count_batches_and_samples():
    dl = DataLoader(_ds(100), 32, shuffle=True, drop_last=False)
    for _ in range(2):
        assert sum(x.shape[0] for x, _ in dl) == 100
    st = dl.stats()
    assert st.batches_loaded == 8 and st.samples_loaded == 200
    assert st.elapsed_s > 0 and st.samples_per_second > 0 and st.avg_wait_ms >= 0
    dl.reset_stats()
    assert dl.stats().batches_loaded == 0


def test_batch_size_optimizer_prefers_fast_sizes_and_respects_memory():
    ds = _ds(1024)

    def step(batch):  # fixed cost per call: larger batches give more samples / s
        time.sleep(0.002)

    res = BatchSizeOptimizer(8, 128, warmup_batches=1, timing_batches=3).find_optimal(ds, step)
    assert [b for b, _ in res.throughput_results] == [8, 16, 32, 64, 128]
    assert res.recommended_batch_size == 128 and not res.memory_limited
    assert all(m == b * (16 * 4 + 8) for b, m in res.memory_results)  # host bytes of one batch
    capped = BatchSizeOptimizer(8, 128, 1, 2).with_max_memory(40 * 72).find_optimal(ds, step)
    assert capped.memory_limited and capped.recommended_batch_size == 32
    assert [b for b, _ in capped.throughput_results] == [8, 16, 32, 64]


def test_memory_aware_loader_sizes_batches_from_budget():
    ds = _ds(1000)
    per_sample = 16 * 4 + 8
    ml = MemoryAwareDataLoader(ds, memory_budget=per_sample * 4 * 100, shuffle=False)
    assert ml.adaptive_batch_size() == 96  # 100 rounded down to a multiple of 8
    assert sum(x.shape[0] for x, _ in ml) == 1000 and len(ml) == 11
    ml.budget = per_sample * 4 * 5
    assert ml.refresh_batch_size() == 5  # below the multiple: kept as is
    assert MemoryAwareDataLoader(ds, memory_budget=1 << 40).adaptive_batch_size() == 1000 - 1000 % 8
    assert MemoryAwareDataLoader(ds, memory_fraction=0.01).adaptive_batch_size() >= 1
