"""Buffer pool reuse and checkpoint-based leak detection (host tensors)."""
import gc

import torch

from scirs_b200.utils import memory as M


def test_buffer_pool_reuses_size_classes():
    pool = M.BufferPool()
    a = pool.acquire(3000)
    assert a.numel() == 3000 and a._base.numel() == 4096
    pool.release(a)
    b = pool.acquire(4000)
    assert b.data_ptr() == a.data_ptr()
    st = pool.stats()
    assert st["hits"] == 1 and st["misses"] == 1
    c = pool.acquire(5000, torch.float16)
    assert c.dtype == torch.float16 and pool.stats()["misses"] == 2


def test_leak_detector_reports_growth():
    det = M.LeakDetector(M.LeakDetectionConfig(capture_stacks=True).with_threshold_mb(0.5))
    keep = []
    det.checkpoint("start")
    for _ in range(4):
        keep.append(det.track(torch.zeros(100_000)))  # 400 KB each, kept alive
    tmp = det.track(torch.zeros(100_000))
    del tmp
    gc.collect()
    rep = det.check("start")
    assert rep.has_leaks() and len(rep.leaks) == 4 and rep.total_leaked_bytes() == 1_600_000
    assert rep.leaks[0].stack and "tracked tensors" in rep.summary()
    keep.clear()
    gc.collect()
    assert not det.check("start").has_leaks()
    assert "host_rss_bytes" in M.memory_usage()
