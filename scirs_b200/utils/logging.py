"""Structured logging with levels, handlers, rate limiting and progress
tracking.

  Logger(name, level, handlers)   entries {time, level, logger, message, fields} go to every
                                  handler: ConsoleLogHandler (text or JSON lines to a stream),
                                  FileLogHandler (JSON lines to a file)
  RateLimiter(strategy)           decides per event key: fixed window, sliding window or token
                                  bucket; CRITICAL / ERROR events bypass it; suppressed counts are
                                  kept per key and reported by `suppression_summary`
  ProgressTracker(name, total)    rate, ETA, percent; reports at most once per update interval

Reference parity: scirs2-core/src/logging.rs:70-520 (LogLevel, LogEntry,
LoggerConfig, Console / File handlers, Logger, ProgressTracker),
logging/rate_limiting.rs:16-680 (RateLimitStrategy, EventClass bypass,
SmartRateLimiter, suppression summaries).
"""
from __future__ import annotations

import json
import sys
import threading
import time
from collections import defaultdict, deque
from dataclasses import dataclass
from enum import IntEnum


class LogLevel(IntEnum):
    TRACE = 0
    DEBUG = 1
    INFO = 2
    WARN = 3
    ERROR = 4
    CRITICAL = 5


class ConsoleLogHandler:
    def __init__(self, stream=None, json_lines: bool = False):
        self.stream = stream if stream is not None else sys.stderr
        self.json_lines = json_lines

    def emit(self, e: dict):
        if self.json_lines:
            self.stream.write(json.dumps(e) + "\n")
        else:
            extra = " ".join(f"{k}={v}" for k, v in e["fields"].items())
            self.stream.write(f"[{e['level']}] {e['logger']}: {e['message']}" + (f" {extra}" if extra else "") + "\n")


class FileLogHandler:
    def __init__(self, path: str):
        self.path = path
        self._lock = threading.Lock()

    def emit(self, e: dict):
        with self._lock, open(self.path, "a") as f:
            f.write(json.dumps(e) + "\n")


@dataclass
class RateLimitStrategy:
    kind: str = "sliding_window"  # fixed_window | sliding_window | token_bucket
    max_events: int = 10
    window_s: float = 60.0
    capacity: int = 10
    refill_per_s: float = 1.0


class RateLimiter:
    def __init__(self, strategy: RateLimitStrategy | None = None, clock=time.monotonic):
        self.s = strategy or RateLimitStrategy()
        if self.s.kind not in ("fixed_window", "sliding_window", "token_bucket"):
            raise ValueError(f"unknown rate-limit strategy {self.s.kind!r}")
        self.clock = clock
        self._events = defaultdict(deque)
        self._window = {}
        self._tokens = {}
        self.suppressed = defaultdict(int)
        self._lock = threading.Lock()

    def allow(self, key: str, level: LogLevel = LogLevel.INFO) -> bool:
        if level >= LogLevel.ERROR:
            return True
        now = self.clock()
        with self._lock:
            s = self.s
            if s.kind == "sliding_window":
                q = self._events[key]
                while q and now - q[0] >= s.window_s:
                    q.popleft()
                ok = len(q) < s.max_events
                if ok:
                    q.append(now)
            elif s.kind == "fixed_window":
                start, n = self._window.get(key, (now, 0))
                if now - start >= s.window_s:
                    start, n = now, 0
                ok = n < s.max_events
                self._window[key] = (start, n + 1 if ok else n)
            else:
                tokens, last = self._tokens.get(key, (float(s.capacity), now))
                tokens = min(float(s.capacity), tokens + (now - last) * s.refill_per_s)
                ok = tokens >= 1.0
                self._tokens[key] = (tokens - 1.0 if ok else tokens, now)
            if not ok:
                self.suppressed[key] += 1
            return ok

    def suppression_summary(self) -> dict:
        return dict(self.suppressed)


class Logger:
    def __init__(self, name: str, level: LogLevel = LogLevel.INFO, handlers=None, rate_limiter: RateLimiter | None = None):
        self.name, self.level = name, level
        self.handlers = list(handlers) if handlers is not None else [ConsoleLogHandler()]
        self.rate_limiter = rate_limiter

    def log(self, level: LogLevel, message: str, **fields):
        if level < self.level:
            return False
        if self.rate_limiter is not None and not self.rate_limiter.allow(f"{self.name}:{message}", level):
            return False
        e = {"time": time.time(), "level": level.name, "logger": self.name, "message": message, "fields": fields}
        for h in self.handlers:
            h.emit(e)
        return True

    def trace(self, m, **f):
        return self.log(LogLevel.TRACE, m, **f)

    def debug(self, m, **f):
        return self.log(LogLevel.DEBUG, m, **f)

    def info(self, m, **f):
        return self.log(LogLevel.INFO, m, **f)

    def warn(self, m, **f):
        return self.log(LogLevel.WARN, m, **f)

    def error(self, m, **f):
        return self.log(LogLevel.ERROR, m, **f)

    def critical(self, m, **f):
        return self.log(LogLevel.CRITICAL, m, **f)


class ProgressTracker:
    def __init__(self, name: str, total: int, logger: Logger | None = None, update_interval_s: float = 1.0,
                 clock=time.monotonic):
        self.name, self.total, self.logger = name, int(total), logger
        self.update_interval_s, self.clock = update_interval_s, clock
        self.start, self.current, self._last_report = clock(), 0, None

    def set_update_interval(self, seconds: float):
        self.update_interval_s = seconds

    def update(self, current: int) -> dict | None:
        self.current = int(current)
        now = self.clock()
        elapsed = max(now - self.start, 1e-12)
        rate = self.current / elapsed
        st = {"name": self.name, "current": self.current, "total": self.total,
              "percent": 100.0 * self.current / self.total if self.total else 100.0, "rate_per_s": rate,
              "eta_s": (self.total - self.current) / rate if rate > 0 else float("inf"), "elapsed_s": elapsed}
        if self._last_report is None or now - self._last_report >= self.update_interval_s or self.current >= self.total:
            self._last_report = now
            if self.logger is not None:
                self.logger.info(f"{self.name} {st['percent']:.1f}%", eta_s=round(st["eta_s"], 2))
            return st
        return None

    def finish(self) -> dict:
        return self.update(self.total)
