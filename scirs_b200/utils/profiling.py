"""Host and device timing, counters and a run-time configuration store.

* `Timer` / `Profiler`: named wall-clock sections with call counts (host); nested
  sections give folded stacks and a flame-graph SVG.
* `SystemMonitor`: background sampling of host CPU / memory and device memory.
* `cuda_timer`: CUDA-event timing of a region on the current stream (the
  synchronise-on-both-sides rule of device timing).
* `Metrics`: counters / gauges / histograms with labels, exportable as
  Prometheus text (prometheus_client is used when installed).
* `Config`: key -> value settings read from `SCIRS_`-prefixed environment
  variables with typed getters.

Reference parity: scirs2-core/src/profiling/profiler.rs:12-290, timer.rs:7-112
(Timer, global Profiler report), metrics.rs:68-350 (Counter / Gauge /
Histogram with labels), config.rs:30-312 (Config with the SCIRS_ prefix).
"""
from __future__ import annotations

import contextlib
import os
import threading
import time
from collections import defaultdict

import torch


class Timer:
    def __init__(self, name: str = ""):
        self.name = name
        self.elapsed = 0.0
        self._t0 = None

    def start(self):
        self._t0 = time.perf_counter()
        return self

    def stop(self) -> float:
        self.elapsed += time.perf_counter() - self._t0
        self._t0 = None
        return self.elapsed

    def __enter__(self):
        return self.start()

    def __exit__(self, *a):
        self.stop()


class Profiler:
    _global = None

    def __init__(self):
        self.totals = defaultdict(float)
        self.calls = defaultdict(int)
        self.stacks = defaultdict(float)  # "outer;inner" -> seconds (nested sections, for flame graphs)
        self._tls = threading.local()
        self._lock = threading.Lock()

    @classmethod
    def global_profiler(cls) -> "Profiler":
        if cls._global is None:
            cls._global = Profiler()
        return cls._global

    @contextlib.contextmanager
    def section(self, name: str):
        stack = getattr(self._tls, "stack", None)
        if stack is None:
            stack = self._tls.stack = []
        stack.append(name)
        path = ";".join(stack)
        t0 = time.perf_counter()
        try:
            yield
        finally:
            dt = time.perf_counter() - t0
            stack.pop()
            with self._lock:
                self.totals[name] += dt
                self.calls[name] += 1
                self.stacks[path] += dt

    def folded(self) -> str:
        """Self time per call stack in the folded format of flame-graph tools ("a;b 123" in us)."""
        lines = []
        for path, t in sorted(self.stacks.items()):
            child = sum(v for p, v in self.stacks.items() if p.startswith(path + ";") and p.count(";") == path.count(";") + 1)
            lines.append(f"{path} {max(0, int(round((t - child) * 1e6)))}")
        return "\n".join(lines)

    def flame_graph_svg(self, path: str, width: int = 1000, row: int = 18) -> str:
        """A flame graph of the nested sections (widths proportional to inclusive time)."""
        roots = {p: t for p, t in self.stacks.items() if ";" not in p}
        total = sum(roots.values()) or 1.0
        rects = []

        def place(prefix, x0, depth):
            kids = sorted((p, t) for p, t in self.stacks.items()
                          if p.startswith(prefix + ";" if prefix else "") and p.count(";") == (prefix.count(";") + 1 if prefix else 0))
            x = x0
            for p, t in kids:
                w = t / total * width
                rects.append((x, depth, w, p.split(";")[-1], t))
                place(p, x, depth + 1)
                x += w

        place("", 0.0, 0)
        depth = max((d for _, d, _, _, _ in rects), default=0) + 1
        h = depth * row
        out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{h}">']
        for x, d, w, name, t in rects:
            y = h - (d + 1) * row
            hue = 20 + (hash(name) % 40)
            out.append(f'<g><title>{name} {t * 1e3:.3f} ms</title><rect x="{x:.2f}" y="{y}" width="{max(w, 0.5):.2f}" '
                       f'height="{row - 1}" fill="hsl({hue},90%,60%)"/>'
                       f'<text x="{x + 2:.2f}" y="{y + row - 5}" font-size="11">{name if w > 40 else ""}</text></g>')
        out.append("</svg>")
        svg = "\n".join(out)
        with open(path, "w") as f:
            f.write(svg)
        return svg

    def report(self) -> str:
        rows = sorted(self.totals.items(), key=lambda kv: -kv[1])
        lines = [f"{'section':40s} {'calls':>8s} {'total ms':>12s} {'mean ms':>10s}"]
        for k, v in rows:
            lines.append(f"{k:40s} {self.calls[k]:8d} {v * 1e3:12.3f} {v * 1e3 / self.calls[k]:10.3f}")
        return "\n".join(lines)

    def reset(self):
        self.totals.clear()
        self.calls.clear()
        self.stacks.clear()


class SystemMonitor:
    """Samples host CPU utilisation and resident memory (psutil) and, when CUDA is available, device
    memory in use, every `interval` seconds on a background thread."""

    def __init__(self, interval: float = 0.5):
        self.interval, self.samples = interval, []
        self._stop = threading.Event()
        self._thread = None

    @staticmethod
    def sample() -> dict:
        import psutil

        proc = psutil.Process()
        d = {"time": time.time(), "cpu_percent": psutil.cpu_percent(interval=None),
             "rss_bytes": proc.memory_info().rss, "host_available_bytes": psutil.virtual_memory().available}
        if torch.cuda.is_available():
            free, total = torch.cuda.mem_get_info()
            d["gpu_used_bytes"], d["gpu_total_bytes"] = total - free, total
        return d

    def start(self):
        self._stop.clear()

        def run():
            while not self._stop.is_set():
                self.samples.append(self.sample())
                self._stop.wait(self.interval)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def stop(self) -> list:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
        return self.samples


@contextlib.contextmanager
def cuda_timer(result: dict, key: str = "ms"):
    """with cuda_timer(d): ... -> d["ms"] = device time of the region."""
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    try:
        yield
    finally:
        e1.record()
        torch.cuda.synchronize()
        result[key] = e0.elapsed_time(e1)


class Metrics:
    """Counters, gauges and histograms with label sets."""

    def __init__(self, buckets=(0.001, 0.01, 0.1, 1.0, 10.0)):
        self.counters = defaultdict(float)
        self.gauges = {}
        self.buckets = tuple(buckets)
        self.hist = {}
        self._lock = threading.Lock()

    @staticmethod
    def _key(name, labels):
        return (name, tuple(sorted((labels or {}).items())))

    def inc(self, name: str, value: float = 1.0, labels: dict | None = None):
        with self._lock:
            self.counters[self._key(name, labels)] += value

    def set(self, name: str, value: float, labels: dict | None = None):
        with self._lock:
            self.gauges[self._key(name, labels)] = value

    def observe(self, name: str, value: float, labels: dict | None = None):
        with self._lock:
            k = self._key(name, labels)
            h = self.hist.setdefault(k, [[0] * (len(self.buckets) + 1), 0.0, 0])
            for i, b in enumerate(self.buckets):
                if value <= b:
                    h[0][i] += 1
            h[0][-1] += 1
            h[1] += value
            h[2] += 1

    def prometheus_text(self) -> str:
        def lab(ls, extra=()):
            items = list(ls) + list(extra)
            return "{" + ",".join(f'{k}="{v}"' for k, v in items) + "}" if items else ""

        out = []
        for (n, ls), v in sorted(self.counters.items()):
            out.append(f"{n}_total{lab(ls)} {v}")
        for (n, ls), v in sorted(self.gauges.items()):
            out.append(f"{n}{lab(ls)} {v}")
        for (n, ls), (cnt, s, c) in sorted(self.hist.items()):
            for b, x in zip(self.buckets + ("+Inf",), cnt):
                out.append(f"{n}_bucket{lab(ls, [('le', b)])} {x}")
            out.append(f"{n}_sum{lab(ls)} {s}")
            out.append(f"{n}_count{lab(ls)} {c}")
        return "\n".join(out) + "\n"


class Config:
    """Settings from `SCIRS_<KEY>` environment variables (or set())."""

    PREFIX = "SCIRS_"

    def __init__(self, env=None):
        self._vals = {}
        env = os.environ if env is None else env
        for k, v in env.items():
            if k.startswith(self.PREFIX):
                self._vals[k[len(self.PREFIX):].lower()] = v

    def set(self, key: str, value):
        self._vals[key.lower()] = value

    def get(self, key: str, default=None):
        return self._vals.get(key.lower(), default)

    def get_int(self, key: str, default: int = 0) -> int:
        v = self.get(key)
        return int(v) if v is not None else default

    def get_float(self, key: str, default: float = 0.0) -> float:
        v = self.get(key)
        return float(v) if v is not None else default

    def get_bool(self, key: str, default: bool = False) -> bool:
        v = self.get(key)
        return default if v is None else str(v).lower() in ("1", "true", "yes", "on")

    def keys(self):
        return list(self._vals)
