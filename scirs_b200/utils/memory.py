"""Memory utilities: a size-class buffer pool, checkpoint-based leak
detection and memory metrics, for host or device tensors.

  BufferPool        reuses freed buffers of the same (size class, dtype,
                    device); sizes round up to powers of two above 1 KiB;
                    hit / miss / bytes statistics
  LeakDetector      `checkpoint(name)` records live bytes (device:
                    torch.cuda.memory_allocated; host: tracked tensors);
                    `check(name)` reports growth above a threshold since the
                    checkpoint, with the tensors (and, optionally, the call
                    stacks) that were allocated through `track` and are still
                    alive
  memory_usage()    current / peak device bytes and host RSS

Reference parity: scirs2-core/src/memory/leak_detection.rs:60-300
(LeakDetectionConfig, MemoryCheckpoint, LeakReport), scirs2-core/src/memory/
buffer pools and metrics.
"""
from __future__ import annotations

import os
import traceback
import weakref
from dataclasses import dataclass, field

import torch


def _size_class(n: int) -> int:
    return n if n <= 256 else 1 << (n - 1).bit_length()


class BufferPool:
    def __init__(self, max_cached_bytes: int = 1 << 30):
        self.max_cached_bytes = max_cached_bytes
        self._free: dict[tuple, list[torch.Tensor]] = {}
        self.cached_bytes = 0
        self.hits = self.misses = 0

    def acquire(self, numel: int, dtype=torch.float32, device="cpu") -> torch.Tensor:
        """A 1-D tensor view of at least `numel` elements (contents undefined)."""
        cls = _size_class(int(numel))
        key = (cls, dtype, torch.device(device))
        lst = self._free.get(key)
        if lst:
            buf = lst.pop()
            self.cached_bytes -= buf.numel() * buf.element_size()
            self.hits += 1
        else:
            buf = torch.empty(cls, dtype=dtype, device=device)
            self.misses += 1
        return buf[:numel]

    def release(self, t: torch.Tensor):
        base = t._base if t._base is not None else t
        nbytes = base.numel() * base.element_size()
        if self.cached_bytes + nbytes > self.max_cached_bytes:
            return
        key = (base.numel(), base.dtype, base.device)
        self._free.setdefault(key, []).append(base)
        self.cached_bytes += nbytes

    def clear(self):
        self._free.clear()
        self.cached_bytes = 0

    def stats(self) -> dict:
        total = self.hits + self.misses
        return {"hits": self.hits, "misses": self.misses, "hit_rate": self.hits / total if total else 0.0,
                "cached_bytes": self.cached_bytes}


@dataclass
class LeakDetectionConfig:
    threshold_bytes: int = 1 << 20
    capture_stacks: bool = False

    def with_threshold_mb(self, mb: float) -> "LeakDetectionConfig":
        self.threshold_bytes = int(mb * (1 << 20))
        return self


@dataclass
class MemoryLeak:
    nbytes: int
    shape: tuple
    dtype: str
    stack: list = field(default_factory=list)


@dataclass
class LeakReport:
    checkpoint: str
    grown_bytes: int
    leaks: list = field(default_factory=list)

    def has_leaks(self) -> bool:
        return bool(self.leaks)

    def total_leaked_bytes(self) -> int:
        return sum(x.nbytes for x in self.leaks)

    def summary(self) -> str:
        return (f"since '{self.checkpoint}': +{self.grown_bytes} bytes, {len(self.leaks)} tracked tensors still "
                f"alive ({self.total_leaked_bytes()} bytes)")


class LeakDetector:
    def __init__(self, config: LeakDetectionConfig | None = None, device=None):
        self.config = config or LeakDetectionConfig()
        self.device = device
        self._checkpoints: dict[str, tuple[int, set]] = {}
        self._tracked: dict[int, tuple] = {}

    def _live_bytes(self) -> int:
        if self.device is not None and torch.device(self.device).type == "cuda":
            return torch.cuda.memory_allocated(self.device)
        return sum(nb for (_, nb, *_rest) in self._tracked.values())

    def track(self, t: torch.Tensor) -> torch.Tensor:
        key = id(t)
        stack = traceback.format_stack()[:-1] if self.config.capture_stacks else []
        ref = weakref.ref(t, lambda _r, k=key: self._tracked.pop(k, None))
        self._tracked[key] = (ref, t.numel() * t.element_size(), tuple(t.shape), str(t.dtype), stack)
        return t

    def checkpoint(self, name: str):
        self._checkpoints[name] = (self._live_bytes(), set(self._tracked))

    def check(self, name: str) -> LeakReport:
        base, ids = self._checkpoints[name]
        grown = self._live_bytes() - base
        leaks = []
        if grown > self.config.threshold_bytes:
            for k, (ref, nb, shape, dt, stack) in list(self._tracked.items()):
                if k not in ids and ref() is not None:
                    leaks.append(MemoryLeak(nb, shape, dt, stack))
        return LeakReport(name, grown, leaks)


def memory_usage(device=None) -> dict:
    out = {}
    if torch.cuda.is_available():
        d = device if device is not None else torch.cuda.current_device()
        out["device_bytes"] = torch.cuda.memory_allocated(d)
        out["device_peak_bytes"] = torch.cuda.max_memory_allocated(d)
    try:
        with open(f"/proc/{os.getpid()}/statm") as f:
            out["host_rss_bytes"] = int(f.read().split()[1]) * os.sysconf("SC_PAGE_SIZE")
    except Exception:
        pass
    return out
