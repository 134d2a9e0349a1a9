"""Observability: distributed tracing (spans with W3C trace-context propagation,
samplers, exporters) and a tamper-evident audit log.

Tracing
  * `TraceContext` carries a 128-bit trace id, a 64-bit span id, the parent span,
    sampling flags, baggage and tracestate; it serialises to / parses from the
    W3C `traceparent` header ("00-<32 hex>-<16 hex>-<2 hex>") and the W3C
    `baggage` header ("k=v,k2=v2", percent-encoded values), so a trace can
    continue in another process or rank.
  * `TracingSystem.start_span` returns an `ActiveSpan` (a context manager);
    spans opened inside it on the same thread become its children. A span
    records attributes, timestamped events, named metrics, a status, host
    wall time and CPU time, and, when `device_timing` is set and CUDA is
    available, the device time between CUDA events recorded on the current
    stream at its start and end (resolved when the spans are exported, so
    timing adds no synchronisation to the traced region). Each span also opens
    an NVTX range, so device profilers show the same names.
  * Samplers decide per trace: `ProbabilitySampler` (by the trace id, so every
    service reaches the same decision), `RateLimitingSampler` (token bucket),
    `AdaptiveSampler` (probability re-tuned each second toward a target rate).
  * Exporters: in-memory, console, JSON lines, Chrome trace-event JSON
    (chrome://tracing / Perfetto; pid = rank), OpenTelemetry OTLP/JSON and a
    batching wrapper.

Audit log
  * `AuditEvent` (category, severity, action, outcome, user / resource ids,
    description, metadata, correlation id, compliance tags, classification,
    system context) built with `AuditEventBuilder`.
  * `AuditLogger` appends JSON lines to rotating files. With the hash chain on,
    each event stores the previous event's hash and its own SHA-256 over its
    canonical JSON; `verify_integrity` re-reads every file, recomputes every
    hash and checks every link, so editing, deleting or reordering a record is
    detected. Search by time window / category / user / action, statistics,
    compliance reports, and an `AlertManager` (threshold counts per category
    in a sliding window, with a cooldown, delivered to callbacks).

Reference parity: scirs2-core/src/observability/tracing.rs:65-1645
(TracingConfig, SpanKind, SpanStatus, TraceContext with traceparent / baggage,
ActiveSpan, SpanBuilder, TracingSystem, samplers, batch / console exporters,
init_tracing / global_tracer, ResourceAttribution) and
observability/audit/{types,builder,logger,storage,alerts}.rs (AuditConfig,
EventCategory / EventSeverity / EventOutcome / DataClassification,
AuditEventBuilder, AuditLogger search / statistics / compliance report /
integrity check, AlertManager). The reference's HTTP exporter, webhook and
e-mail alerts are callbacks here (there is no network on a training node's
critical path); its hash covers a fixed list of fields, this one the whole
canonical record.
"""
from __future__ import annotations

import contextlib
import dataclasses
import enum
import hashlib
import json
import os
import secrets
import socket
import sys
import threading
import time
import urllib.parse
import uuid
from collections import defaultdict, deque
from datetime import datetime, timedelta, timezone
from typing import Callable

import torch

# ============================================================================ tracing


@dataclasses.dataclass
class TracingConfig:
    service_name: str = "scirs_b200"
    service_version: str = "0.1.0"
    environment: str = "production"
    sampling_rate: float = 1.0
    max_active_spans: int = 10_000
    span_timeout_s: float = 300.0
    default_attributes: dict = dataclasses.field(default_factory=dict)
    export_batch_size: int = 100
    device_timing: bool = False  # CUDA-event device time per span
    nvtx: bool = True


class SpanKind(enum.Enum):
    INTERNAL = "internal"
    SERVER = "server"
    CLIENT = "client"
    PRODUCER = "producer"
    CONSUMER = "consumer"


class SpanStatus(enum.Enum):
    UNSET = "unset"
    OK = "ok"
    ERROR = "error"


def _hex_id(nbytes: int) -> str:
    while True:
        h = secrets.token_hex(nbytes)
        if int(h, 16):  # all-zero ids are invalid in the W3C format
            return h


@dataclasses.dataclass
class TraceContext:
    trace_id: str = dataclasses.field(default_factory=lambda: _hex_id(16))
    span_id: str = dataclasses.field(default_factory=lambda: _hex_id(8))
    parent_span_id: str | None = None
    trace_flags: int = 1  # bit 0: sampled
    baggage: dict = dataclasses.field(default_factory=dict)
    tracestate: str | None = None
    is_remote: bool = False

    def child(self) -> "TraceContext":
        return TraceContext(self.trace_id, _hex_id(8), self.span_id, self.trace_flags, dict(self.baggage),
                            self.tracestate, False)

    def remote_child(self) -> "TraceContext":
        c = self.child()
        c.is_remote = True
        return c

    @property
    def is_sampled(self) -> bool:
        return bool(self.trace_flags & 1)

    def with_baggage(self, key: str, value: str) -> "TraceContext":
        self.baggage[key] = value
        return self

    def with_tracestate(self, tracestate: str) -> "TraceContext":
        self.tracestate = tracestate
        return self

    def to_traceparent(self) -> str:
        return f"00-{self.trace_id}-{self.span_id}-{self.trace_flags:02x}"

    @classmethod
    def from_traceparent(cls, header: str) -> "TraceContext":
        parts = header.strip().split("-")
        if len(parts) != 4 or parts[0] != "00":
            raise ValueError(f"invalid traceparent header: {header!r}")
        _, tid, sid, flags = parts
        ok = (len(tid) == 32 and len(sid) == 16 and len(flags) == 2
              and all(c in "0123456789abcdef" for c in tid + sid + flags))
        if not ok or int(tid, 16) == 0 or int(sid, 16) == 0:
            raise ValueError(f"invalid traceparent header: {header!r}")
        # the header names the caller's span: it becomes the parent of the local span
        return cls(tid, _hex_id(8), sid, int(flags, 16), {}, None, True)

    def to_baggage(self) -> str | None:
        if not self.baggage:
            return None
        return ",".join(f"{urllib.parse.quote(k, safe='')}={urllib.parse.quote(str(v), safe='')}"
                        for k, v in sorted(self.baggage.items()))

    def with_baggage_header(self, header: str) -> "TraceContext":
        for item in header.split(","):
            kv = item.split(";")[0].strip()  # drop W3C baggage properties
            if "=" in kv:
                k, v = kv.split("=", 1)
                self.baggage[urllib.parse.unquote(k.strip())] = urllib.parse.unquote(v.strip())
        return self

    def headers(self) -> dict:
        h = {"traceparent": self.to_traceparent()}
        if self.tracestate:
            h["tracestate"] = self.tracestate
        b = self.to_baggage()
        if b:
            h["baggage"] = b
        return h

    @classmethod
    def from_headers(cls, headers: dict) -> "TraceContext":
        ctx = cls.from_traceparent(headers["traceparent"])
        if headers.get("tracestate"):
            ctx.tracestate = headers["tracestate"]
        if headers.get("baggage"):
            ctx.with_baggage_header(headers["baggage"])
        return ctx


@dataclasses.dataclass
class ResourceAttribution:
    cpu_time_ns: int = 0
    memory_bytes: int = 0
    io_operations: int = 0
    bytes_read: int = 0
    bytes_written: int = 0
    gpu_memory_bytes: int = 0
    gpu_time_ns: int = 0

    def merge(self, other: "ResourceAttribution") -> None:
        for f in dataclasses.fields(self):
            if f.name in ("memory_bytes", "gpu_memory_bytes"):
                setattr(self, f.name, max(getattr(self, f.name), getattr(other, f.name)))  # peaks
            else:
                setattr(self, f.name, getattr(self, f.name) + getattr(other, f.name))


@dataclasses.dataclass
class SpanEvent:
    name: str
    time_ns: int
    attributes: dict


@dataclasses.dataclass
class Span:
    name: str
    context: TraceContext
    kind: SpanKind
    start_ns: int
    end_ns: int | None = None
    attributes: dict = dataclasses.field(default_factory=dict)
    events: list = dataclasses.field(default_factory=list)
    metrics: dict = dataclasses.field(default_factory=dict)
    status: SpanStatus = SpanStatus.UNSET
    error: str | None = None
    component: str | None = None
    thread_id: int = 0
    resources: ResourceAttribution = dataclasses.field(default_factory=ResourceAttribution)
    _cuda_events: tuple | None = None

    @property
    def duration_ns(self) -> int | None:
        return None if self.end_ns is None else self.end_ns - self.start_ns

    def resolve_device_time(self) -> None:
        """Device time between the span's CUDA events (waits for the end event)."""
        if self._cuda_events is not None:
            e0, e1 = self._cuda_events
            e1.synchronize()
            self.resources.gpu_time_ns = int(e0.elapsed_time(e1) * 1e6)
            self.metrics["device_ms"] = e0.elapsed_time(e1)
            self._cuda_events = None

    def to_dict(self) -> dict:
        return {
            "name": self.name, "trace_id": self.context.trace_id, "span_id": self.context.span_id,
            "parent_span_id": self.context.parent_span_id, "kind": self.kind.value, "start_ns": self.start_ns,
            "end_ns": self.end_ns, "duration_ns": self.duration_ns, "attributes": self.attributes,
            "events": [dataclasses.asdict(e) for e in self.events], "metrics": self.metrics,
            "status": self.status.value, "error": self.error, "component": self.component,
            "baggage": self.context.baggage, "resources": dataclasses.asdict(self.resources),
        }


class ActiveSpan:
    """An open span; use as a context manager (`with tracer.start_span("step") as s:`)."""

    def __init__(self, system: "TracingSystem", span: Span, sampled: bool):
        self._sys, self.span, self.sampled = system, span, sampled
        self._lock = threading.Lock()
        self._ended = False
        self._cpu0 = time.thread_time_ns()
        self._nvtx = False

    def _begin(self):
        cfg = self._sys.config
        if self.sampled and cfg.device_timing and torch.cuda.is_available():
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            self.span._cuda_events = (e0, e1)
        if self.sampled and cfg.nvtx and torch.cuda.is_available():
            torch.cuda.nvtx.range_push(self.span.name)
            self._nvtx = True
        return self

    @property
    def context(self) -> TraceContext:
        return self.span.context

    def add_attribute(self, key: str, value) -> "ActiveSpan":
        with self._lock:
            self.span.attributes[key] = value
        return self

    def add_event(self, name: str, attributes: dict | None = None) -> "ActiveSpan":
        with self._lock:
            self.span.events.append(SpanEvent(name, time.time_ns(), dict(attributes or {})))
        return self

    def add_metric(self, name: str, value: float) -> "ActiveSpan":
        with self._lock:
            self.span.metrics[name] = float(value)
        return self

    def set_status(self, status: SpanStatus) -> "ActiveSpan":
        self.span.status = status
        return self

    def set_error(self, error: str) -> "ActiveSpan":
        self.span.status, self.span.error = SpanStatus.ERROR, error
        return self

    def in_span(self, fn: Callable, *args, **kwargs):
        """Runs fn with this span current; an exception marks the span as failed."""
        with self._sys._activate(self):
            try:
                return fn(*args, **kwargs)
            except Exception as e:
                self.set_error(repr(e))
                raise

    def end(self) -> None:
        if self._ended:
            return
        self._ended = True
        if self.span._cuda_events is not None:
            self.span._cuda_events[1].record()
        if self._nvtx:
            torch.cuda.nvtx.range_pop()
        self.span.end_ns = time.time_ns()
        self.span.resources.cpu_time_ns += time.thread_time_ns() - self._cpu0
        if self.span.status == SpanStatus.UNSET:
            self.span.status = SpanStatus.OK
        self._sys._finish(self)

    def __enter__(self):
        self._sys._push(self)
        return self

    def __exit__(self, et, ev, tb):
        if ev is not None:
            self.set_error(repr(ev))
        self._sys._pop(self)
        self.end()
        return False


class SpanBuilder:
    def __init__(self, name: str):
        self.name, self.kind, self.attributes = name, SpanKind.INTERNAL, {}
        self.parent: TraceContext | None = None
        self.component: str | None = None

    def with_kind(self, kind: SpanKind) -> "SpanBuilder":
        self.kind = kind
        return self

    def with_attribute(self, key: str, value) -> "SpanBuilder":
        self.attributes[key] = value
        return self

    def with_parent(self, context: TraceContext) -> "SpanBuilder":
        self.parent = context
        return self

    def with_component(self, component: str) -> "SpanBuilder":
        self.component = component
        return self

    def start(self, system: "TracingSystem") -> ActiveSpan:
        return system.start_span_with_builder(self)


# ---------------------------------------------------------------------------- samplers


class ProbabilitySampler:
    """Samples a trace iff the low 64 bits of its id, as a fraction of 2^64, are below the rate."""

    def __init__(self, rate: float):
        self.rate = min(1.0, max(0.0, rate))

    def should_sample(self, ctx: TraceContext) -> bool:
        return int(ctx.trace_id[16:], 16) / 2.0**64 < self.rate


class RateLimitingSampler:
    """At most `max_per_second` sampled traces per second (token bucket of one second's capacity)."""

    def __init__(self, max_per_second: float, clock: Callable[[], float] = time.monotonic):
        self.rate, self._clock = float(max_per_second), clock
        self._tokens, self._t = float(max_per_second), clock()
        self._lock = threading.Lock()

    def should_sample(self, ctx: TraceContext) -> bool:
        with self._lock:
            now = self._clock()
            self._tokens = min(self.rate, self._tokens + (now - self._t) * self.rate)
            self._t = now
            if self._tokens >= 1.0:
                self._tokens -= 1.0
                return True
            return False


class AdaptiveSampler:
    """Probability sampling whose rate is re-tuned once per second so that the sampled traces per second
    approach `target_per_second` (rate = target / observed traces per second, clamped to
    [min_rate, 1])."""

    def __init__(self, base_rate: float, target_per_second: float, min_rate: float = 1e-4,
                 clock: Callable[[], float] = time.monotonic):
        self.rate, self.target, self.min_rate, self._clock = base_rate, target_per_second, min_rate, clock
        self._window_start, self._seen = clock(), 0
        self.total_seen = self.total_sampled = 0
        self._lock = threading.Lock()

    def should_sample(self, ctx: TraceContext) -> bool:
        with self._lock:
            now = self._clock()
            if now - self._window_start >= 1.0:
                per_s = self._seen / (now - self._window_start)
                if per_s > 0:
                    self.rate = min(1.0, max(self.min_rate, self.target / per_s))
                self._window_start, self._seen = now, 0
            self._seen += 1
            self.total_seen += 1
            hit = ProbabilitySampler(self.rate).should_sample(ctx)
            self.total_sampled += hit
            return hit

    def get_stats(self) -> tuple[int, int, float]:
        return self.total_seen, self.total_sampled, self.rate


# ---------------------------------------------------------------------------- exporters


class InMemoryExporter:
    def __init__(self):
        self.spans: list[Span] = []

    def export(self, spans: list[Span]) -> None:
        self.spans.extend(spans)


class ConsoleExporter:
    def __init__(self, pretty: bool = False, stream=None):
        self.pretty, self.stream = pretty, stream or sys.stderr

    def export(self, spans: list[Span]) -> None:
        for s in spans:
            print(json.dumps(s.to_dict(), indent=2 if self.pretty else None, default=str), file=self.stream)


class JsonlExporter:
    def __init__(self, path: str):
        self.path = path

    def export(self, spans: list[Span]) -> None:
        with open(self.path, "a") as f:
            for s in spans:
                f.write(json.dumps(s.to_dict(), default=str) + "\n")


class ChromeTraceExporter:
    """Trace-event JSON ("X" complete events; pid = rank, tid = thread) for chrome://tracing / Perfetto.
    `write()` produces the file from everything exported so far."""

    def __init__(self, path: str, rank: int | None = None):
        self.path = path
        self.rank = rank if rank is not None else int(os.environ.get("RANK", "0"))
        self.events: list[dict] = []

    def export(self, spans: list[Span]) -> None:
        for s in spans:
            args = dict(s.attributes)
            args.update({f"metric.{k}": v for k, v in s.metrics.items()})
            self.events.append({"name": s.name, "ph": "X", "ts": s.start_ns / 1e3, "dur": (s.duration_ns or 0) / 1e3,
                                "pid": self.rank, "tid": s.thread_id, "cat": s.component or s.kind.value,
                                "args": args})
            for e in s.events:
                self.events.append({"name": e.name, "ph": "i", "s": "t", "ts": e.time_ns / 1e3, "pid": self.rank,
                                    "tid": s.thread_id, "args": e.attributes})

    def write(self) -> str:
        with open(self.path, "w") as f:
            json.dump({"traceEvents": self.events, "displayTimeUnit": "ms"}, f)
        return self.path


def _otlp_value(v) -> dict:
    if isinstance(v, bool):
        return {"boolValue": v}
    if isinstance(v, int):
        return {"intValue": str(v)}  # 64-bit integers are strings in OTLP/JSON
    if isinstance(v, float):
        return {"doubleValue": v}
    return {"stringValue": str(v)}


def _otlp_attrs(d: dict) -> list:
    return [{"key": str(k), "value": _otlp_value(v)} for k, v in d.items()]


_OTLP_KIND = {SpanKind.INTERNAL: 1, SpanKind.SERVER: 2, SpanKind.CLIENT: 3, SpanKind.PRODUCER: 4,
              SpanKind.CONSUMER: 5}
_OTLP_STATUS = {SpanStatus.UNSET: 0, SpanStatus.OK: 1, SpanStatus.ERROR: 2}


class OtlpJsonExporter:
    """OpenTelemetry OTLP/JSON trace documents (resourceSpans -> scopeSpans -> spans, hex ids, times in
    Unix nanoseconds as strings, typed attribute values), one document per export appended as a line
    to `path`, the file format OpenTelemetry collectors' file receivers read. Span metrics become
    attributes named `metric.<name>`."""

    def __init__(self, path: str, service_name: str = "scirs_b200", resource: dict | None = None):
        self.path, self.resource = path, {"service.name": service_name, **(resource or {})}

    def document(self, spans: list[Span]) -> dict:
        out = []
        for s in spans:
            attrs = dict(s.attributes)
            attrs.update({f"metric.{k}": v for k, v in s.metrics.items()})
            d = {"traceId": s.context.trace_id, "spanId": s.context.span_id, "name": s.name,
                 "kind": _OTLP_KIND[s.kind], "startTimeUnixNano": str(s.start_ns),
                 "endTimeUnixNano": str(s.end_ns or s.start_ns), "attributes": _otlp_attrs(attrs),
                 "events": [{"timeUnixNano": str(e.time_ns), "name": e.name, "attributes": _otlp_attrs(e.attributes)}
                            for e in s.events],
                 "status": {"code": _OTLP_STATUS[s.status], **({"message": s.error} if s.error else {})}}
            if s.context.parent_span_id:
                d["parentSpanId"] = s.context.parent_span_id
            out.append(d)
        return {"resourceSpans": [{"resource": {"attributes": _otlp_attrs(self.resource)},
                                   "scopeSpans": [{"scope": {"name": "scirs_b200.observability"},
                                                   "spans": out}]}]}

    def export(self, spans: list[Span]) -> None:
        with open(self.path, "a") as f:
            f.write(json.dumps(self.document(spans)) + "\n")


class BatchExporter:
    """Buffers finished spans and hands them to `inner` in batches of `batch_size` (and on flush)."""

    def __init__(self, inner, batch_size: int = 100):
        self.inner, self.batch_size = inner, max(1, batch_size)
        self._buf: list[Span] = []
        self._lock = threading.Lock()
        self.batches_sent = 0

    def export(self, spans: list[Span]) -> None:
        with self._lock:
            self._buf.extend(spans)
            while len(self._buf) >= self.batch_size:
                batch, self._buf = self._buf[: self.batch_size], self._buf[self.batch_size:]
                self.inner.export(batch)
                self.batches_sent += 1

    def flush(self) -> None:
        with self._lock:
            if self._buf:
                self.inner.export(self._buf)
                self.batches_sent += 1
                self._buf = []


# ---------------------------------------------------------------------------- tracing system


@dataclasses.dataclass
class TracingMetrics:
    spans_started: int = 0
    spans_finished: int = 0
    spans_dropped: int = 0
    spans_not_sampled: int = 0
    spans_exported: int = 0
    active_spans: int = 0


class TracingSystem:
    def __init__(self, config: TracingConfig | None = None, exporter=None, sampler=None):
        self.config = config or TracingConfig()
        self.exporter = exporter if exporter is not None else InMemoryExporter()
        self.sampler = sampler if sampler is not None else ProbabilitySampler(self.config.sampling_rate)
        self._tls = threading.local()
        self._active: dict[str, ActiveSpan] = {}
        self._pending: list[Span] = []
        self._lock = threading.Lock()
        self.metrics = TracingMetrics()

    def with_exporter(self, exporter) -> "TracingSystem":
        self.exporter = exporter
        return self

    # current-span stack per thread
    def _stack(self) -> list:
        st = getattr(self._tls, "stack", None)
        if st is None:
            st = self._tls.stack = []
        return st

    def _push(self, s: ActiveSpan):
        self._stack().append(s)

    def _pop(self, s: ActiveSpan):
        st = self._stack()
        if st and st[-1] is s:
            st.pop()
        elif s in st:
            st.remove(s)

    @contextlib.contextmanager
    def _activate(self, s: ActiveSpan):
        self._push(s)
        try:
            yield
        finally:
            self._pop(s)

    def current_span(self) -> ActiveSpan | None:
        st = self._stack()
        return st[-1] if st else None

    def start_span(self, name: str, kind: SpanKind = SpanKind.INTERNAL, attributes: dict | None = None,
                   parent: TraceContext | None = None, component: str | None = None) -> ActiveSpan:
        b = SpanBuilder(name).with_kind(kind).with_component(component)
        b.attributes.update(attributes or {})
        if parent is not None:
            b.with_parent(parent)
        return self.start_span_with_builder(b)

    def start_span_with_builder(self, b: SpanBuilder) -> ActiveSpan:
        if b.parent is not None:
            # a remote context (parsed from a header) already names the caller's span as parent
            ctx = b.parent if b.parent.is_remote and b.parent.parent_span_id else b.parent.child()
        else:
            cur = self.current_span()
            ctx = cur.context.child() if cur is not None else TraceContext()
        if b.parent is None and self.current_span() is None:
            ctx.trace_flags = 1 if self.sampler.should_sample(ctx) else 0
        sampled = ctx.is_sampled
        attrs = dict(self.config.default_attributes)
        attrs.update({"service.name": self.config.service_name, "service.version": self.config.service_version,
                      "deployment.environment": self.config.environment})
        attrs.update(b.attributes)
        span = Span(b.name, ctx, b.kind, time.time_ns(), attributes=attrs, component=b.component,
                    thread_id=threading.get_ident() & 0xFFFF)
        a = ActiveSpan(self, span, sampled)
        with self._lock:
            self.metrics.spans_started += 1
            if not sampled:
                self.metrics.spans_not_sampled += 1
            elif len(self._active) >= self.config.max_active_spans:
                self.metrics.spans_dropped += 1
                a.sampled = False
            else:
                self._active[ctx.span_id] = a
            self.metrics.active_spans = len(self._active)
        return a._begin()

    def _finish(self, a: ActiveSpan):
        with self._lock:
            self._active.pop(a.span.context.span_id, None)
            self.metrics.active_spans = len(self._active)
            self.metrics.spans_finished += 1
            if a.sampled:
                self._pending.append(a.span)
                ready = len(self._pending) >= self.config.export_batch_size and not any(
                    s._cuda_events for s in self._pending)
            else:
                ready = False
        if ready:
            self.flush()

    def record_span(self, span: Span) -> None:
        """Adds a span finished elsewhere (e.g. received from another rank)."""
        with self._lock:
            self._pending.append(span)

    def cleanup_expired_spans(self) -> int:
        """Ends spans open longer than the span timeout (marked as errors); returns how many."""
        limit = time.time_ns() - int(self.config.span_timeout_s * 1e9)
        with self._lock:
            stale = [a for a in self._active.values() if a.span.start_ns < limit]
        for a in stale:
            a.set_error("span timed out")
            a.end()
        return len(stale)

    def get_metrics(self) -> TracingMetrics:
        with self._lock:
            return dataclasses.replace(self.metrics)

    def flush(self) -> int:
        with self._lock:
            batch, self._pending = self._pending, []
        for s in batch:
            s.resolve_device_time()
        if batch:
            self.exporter.export(batch)
        if hasattr(self.exporter, "flush"):
            self.exporter.flush()
        with self._lock:
            self.metrics.spans_exported += len(batch)
        return len(batch)


_GLOBAL: TracingSystem | None = None


def init_tracing(config: TracingConfig | None = None, exporter=None, sampler=None) -> TracingSystem:
    global _GLOBAL
    _GLOBAL = TracingSystem(config, exporter, sampler)
    return _GLOBAL


def global_tracer() -> TracingSystem | None:
    return _GLOBAL


def traced(name: str | None = None, tracer: TracingSystem | None = None):
    """Decorator: runs the function inside a span of the given (or global) tracer."""

    def wrap(fn):
        def inner(*a, **k):
            t = tracer or _GLOBAL
            if t is None:
                return fn(*a, **k)
            with t.start_span(name or fn.__qualname__):
                return fn(*a, **k)

        inner.__wrapped__ = fn
        inner.__name__ = fn.__name__
        return inner

    return wrap


# ============================================================================ audit log


class EventCategory(enum.Enum):
    AUTHENTICATION = "authentication"
    AUTHORIZATION = "authorization"
    DATA_ACCESS = "data_access"
    CONFIGURATION = "configuration"
    SECURITY = "security"
    PERFORMANCE = "performance"
    ERROR = "error"
    ADMINISTRATIVE = "administrative"
    COMPLIANCE = "compliance"


class EventSeverity(enum.IntEnum):
    INFO = 0
    WARNING = 1
    ERROR = 2
    CRITICAL = 3


class EventOutcome(enum.Enum):
    SUCCESS = "success"
    FAILURE = "failure"
    DENIED = "denied"
    CANCELLED = "cancelled"
    UNKNOWN = "unknown"


class DataClassification(enum.IntEnum):
    PUBLIC = 0
    INTERNAL = 1
    CONFIDENTIAL = 2
    RESTRICTED = 3
    TOP_SECRET = 4


class ComplianceMode(enum.Enum):
    STANDARD = "standard"
    FINANCIAL = "financial"
    HEALTHCARE = "healthcare"
    DATA_PROTECTION = "data_protection"
    GOVERNMENT = "government"


def _now() -> datetime:
    return datetime.now(timezone.utc)


def system_context() -> dict:
    return {"process_id": os.getpid(), "hostname": socket.gethostname(), "rank": int(os.environ.get("RANK", "0")),
            "thread_id": threading.get_ident()}


@dataclasses.dataclass
class AuditEvent:
    category: EventCategory
    action: str
    severity: EventSeverity = EventSeverity.INFO
    outcome: EventOutcome = EventOutcome.SUCCESS
    description: str = ""
    user_id: str | None = None
    resource_id: str | None = None
    source_ip: str | None = None
    metadata: dict = dataclasses.field(default_factory=dict)
    correlation_id: str | None = None
    compliance_tags: list = dataclasses.field(default_factory=list)
    data_classification: DataClassification | None = None
    system_context: dict | None = None
    event_id: str = dataclasses.field(default_factory=lambda: str(uuid.uuid4()))
    timestamp: str = dataclasses.field(default_factory=lambda: _now().isoformat())
    previous_hash: str | None = None
    hash: str | None = None

    def to_dict(self) -> dict:
        d = dataclasses.asdict(self)
        d["category"] = self.category.value
        d["severity"] = self.severity.name.lower()
        d["outcome"] = self.outcome.value
        d["data_classification"] = None if self.data_classification is None else self.data_classification.name.lower()
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "AuditEvent":
        d = dict(d)
        d["category"] = EventCategory(d["category"])
        d["severity"] = EventSeverity[d["severity"].upper()]
        d["outcome"] = EventOutcome(d["outcome"])
        if d.get("data_classification") is not None:
            d["data_classification"] = DataClassification[d["data_classification"].upper()]
        return cls(**d)

    def canonical_hash(self) -> str:
        d = self.to_dict()
        d.pop("hash")
        return hashlib.sha256(json.dumps(d, sort_keys=True, separators=(",", ":"), default=str).encode()).hexdigest()

    @property
    def time(self) -> datetime:
        return datetime.fromisoformat(self.timestamp)


class AuditEventBuilder:
    def __init__(self, category: EventCategory, action: str):
        self._e = AuditEvent(category, action)

    def severity(self, s: EventSeverity):
        self._e.severity = s
        return self

    def outcome(self, o: EventOutcome):
        self._e.outcome = o
        return self

    def user_id(self, u: str):
        self._e.user_id = u
        return self

    def resource_id(self, r: str):
        self._e.resource_id = r
        return self

    def source_ip(self, ip: str):
        self._e.source_ip = ip
        return self

    def description(self, d: str):
        self._e.description = d
        return self

    def metadata(self, key: str, value):
        self._e.metadata[key] = value
        return self

    def system_context(self, ctx: dict | None = None):
        self._e.system_context = ctx if ctx is not None else system_context()
        return self

    def correlation_id(self, cid: str):
        self._e.correlation_id = cid
        return self

    def data_classification(self, c: DataClassification):
        self._e.data_classification = c
        return self

    def compliance_tag(self, tag: str):
        self._e.compliance_tags.append(tag)
        return self

    def build(self) -> AuditEvent:
        return self._e


@dataclasses.dataclass
class AlertingConfig:
    enabled: bool = True
    failed_auth_threshold: int = 5
    data_access_rate_threshold: int = 1000
    config_change_threshold: int = 10
    window_s: float = 60.0
    cooldown_s: float = 300.0


class AlertManager:
    """Counts events per alert kind in a sliding window; past a threshold it calls every handler with
    (alert_key, event), then stays quiet for the cooldown."""

    def __init__(self, config: AlertingConfig | None = None, clock: Callable[[], float] = time.monotonic):
        self.config = config or AlertingConfig()
        self.handlers: list[Callable[[str, AuditEvent], None]] = []
        self._clock = clock
        self._times: dict[str, deque] = defaultdict(deque)
        self._last_alert: dict[str, float] = {}
        self.sent: list[tuple[str, str]] = []

    def add_handler(self, fn: Callable[[str, AuditEvent], None]) -> None:
        self.handlers.append(fn)

    def _key_threshold(self, e: AuditEvent):
        c = self.config
        if e.category == EventCategory.AUTHENTICATION and e.outcome in (EventOutcome.FAILURE, EventOutcome.DENIED):
            return "failed_authentication", c.failed_auth_threshold
        if e.category == EventCategory.DATA_ACCESS:
            return "data_access_rate", c.data_access_rate_threshold
        if e.category == EventCategory.CONFIGURATION:
            return "configuration_changes", c.config_change_threshold
        if e.severity == EventSeverity.CRITICAL:
            return "critical_event", 1
        return None, 0

    def process_event(self, e: AuditEvent) -> bool:
        if not self.config.enabled:
            return False
        key, thr = self._key_threshold(e)
        if key is None:
            return False
        now = self._clock()
        q = self._times[key]
        q.append(now)
        while q and now - q[0] > self.config.window_s:
            q.popleft()
        if len(q) < thr:
            return False
        last = self._last_alert.get(key)
        if last is not None and now - last < self.config.cooldown_s:
            return False
        self._last_alert[key] = now
        self.sent.append((key, e.event_id))
        for h in self.handlers:
            h(key, e)
        return True


@dataclasses.dataclass
class AuditConfig:
    log_directory: str = "./auditlogs"
    max_file_size: int = 100 * 1024 * 1024
    max_files: int = 100
    buffer_size: int = 1000
    enable_hash_chain: bool = True
    include_system_context: bool = True
    compliance_mode: ComplianceMode = ComplianceMode.STANDARD
    alerting: AlertingConfig | None = None


class AuditLogger:
    """Append-only audit log in `audit_<n>.log` JSON-lines files (rotated by size, at most max_files)."""

    def __init__(self, config: AuditConfig | None = None):
        self.config = config or AuditConfig()
        os.makedirs(self.config.log_directory, exist_ok=True)
        self._lock = threading.Lock()
        self._buf: list[AuditEvent] = []
        self.alerts = AlertManager(self.config.alerting) if self.config.alerting else None
        files = self._files()
        self._seq = int(files[-1].rsplit("_", 1)[1].split(".")[0]) if files else 0
        self._last_hash = self._read_last_hash(files)

    # ---- files
    def _files(self) -> list[str]:
        d = self.config.log_directory
        names = [n for n in os.listdir(d) if n.startswith("audit_") and n.endswith(".log")]
        return [os.path.join(d, n) for n in sorted(names, key=lambda n: int(n[6:-4]))]

    def _path(self) -> str:
        return os.path.join(self.config.log_directory, f"audit_{self._seq:06d}.log")

    @staticmethod
    def _read_last_hash(files: list[str]) -> str | None:
        for p in reversed(files):
            with open(p) as f:
                lines = [ln for ln in f if ln.strip()]
            if lines:
                return json.loads(lines[-1]).get("hash")
        return None

    # ---- writing
    def log_event(self, event: AuditEvent) -> AuditEvent:
        if self.config.include_system_context and event.system_context is None:
            event.system_context = system_context()
        with self._lock:
            if self.config.enable_hash_chain:
                event.previous_hash = self._last_hash
                event.hash = event.canonical_hash()
                self._last_hash = event.hash
            self._buf.append(event)
            full = len(self._buf) >= self.config.buffer_size
        if full:
            self.flush()
        if self.alerts is not None:
            self.alerts.process_event(event)
        return event

    def log_data_access(self, user_id: str, resource_id: str, action: str, outcome=EventOutcome.SUCCESS,
                        description: str = "") -> AuditEvent:
        return self.log_event(AuditEventBuilder(EventCategory.DATA_ACCESS, action).user_id(user_id)
                              .resource_id(resource_id).outcome(outcome).description(description).build())

    def log_security_event(self, action: str, severity: EventSeverity, description: str,
                           user_id: str | None = None) -> AuditEvent:
        b = AuditEventBuilder(EventCategory.SECURITY, action).severity(severity).description(description)
        if user_id:
            b.user_id(user_id)
        return self.log_event(b.build())

    def log_authentication(self, user_id: str, success: bool, method: str = "password",
                           source_ip: str | None = None) -> AuditEvent:
        b = (AuditEventBuilder(EventCategory.AUTHENTICATION, "login").user_id(user_id)
             .outcome(EventOutcome.SUCCESS if success else EventOutcome.FAILURE)
             .severity(EventSeverity.INFO if success else EventSeverity.WARNING).metadata("method", method))
        if source_ip:
            b.source_ip(source_ip)
        return self.log_event(b.build())

    def log_configuration_change(self, user_id: str, key: str, old_value, new_value) -> AuditEvent:
        return self.log_event(AuditEventBuilder(EventCategory.CONFIGURATION, "config_change").user_id(user_id)
                              .resource_id(key).metadata("old_value", old_value).metadata("new_value", new_value)
                              .severity(EventSeverity.WARNING).build())

    def flush(self) -> None:
        with self._lock:
            buf, self._buf = self._buf, []
            if not buf:
                return
            f = open(self._path(), "a")  # noqa: SIM115 - replaced on rotation, closed below
            try:
                for e in buf:
                    if f.tell() >= self.config.max_file_size:
                        f.close()
                        self._seq += 1
                        f = open(self._path(), "a")  # noqa: SIM115
                    f.write(json.dumps(e.to_dict(), default=str) + "\n")
            finally:
                f.close()
            self._enforce_max_files()

    def _enforce_max_files(self) -> None:
        files = self._files()
        for p in files[: max(0, len(files) - self.config.max_files)]:
            os.remove(p)

    # ---- reading
    def _read_all(self) -> list[AuditEvent]:
        self.flush()
        out = []
        for p in self._files():
            with open(p) as f:
                out.extend(AuditEvent.from_dict(json.loads(ln)) for ln in f if ln.strip())
        return out

    def search_events(self, start: datetime | None = None, end: datetime | None = None,
                      category: EventCategory | None = None, user_id: str | None = None,
                      action: str | None = None, limit: int | None = None) -> list[AuditEvent]:
        res = []
        for e in self._read_all():
            t = e.time
            if (start and t < start) or (end and t > end) or (category and e.category != category):
                continue
            if (user_id and e.user_id != user_id) or (action and action not in e.action):
                continue
            res.append(e)
            if limit and len(res) >= limit:
                break
        return res

    def get_statistics(self, days: int = 1) -> dict:
        evs = self.search_events(start=_now() - timedelta(days=days))
        by_cat, by_sev, by_out, users = defaultdict(int), defaultdict(int), defaultdict(int), set()
        for e in evs:
            by_cat[e.category.value] += 1
            by_sev[e.severity.name.lower()] += 1
            by_out[e.outcome.value] += 1
            if e.user_id:
                users.add(e.user_id)
        return {"total_events": len(evs), "by_category": dict(by_cat), "by_severity": dict(by_sev),
                "by_outcome": dict(by_out), "unique_users": len(users)}

    def export_compliance_report(self, start: datetime, end: datetime,
                                 mode: ComplianceMode | None = None) -> dict:
        evs = self.search_events(start, end)
        cats = defaultdict(int)
        for e in evs:
            cats[e.category.value] += 1
        return {
            "period_start": start.isoformat(), "period_end": end.isoformat(),
            "compliance_mode": (mode or self.config.compliance_mode).value, "total_events": len(evs),
            "events_by_category": dict(cats),
            "security_violations": sum(e.category == EventCategory.SECURITY and e.outcome == EventOutcome.FAILURE
                                       for e in evs),
            "failed_authentications": sum(e.category == EventCategory.AUTHENTICATION
                                          and e.outcome != EventOutcome.SUCCESS for e in evs),
            "data_access_events": cats[EventCategory.DATA_ACCESS.value],
            "configuration_changes": cats[EventCategory.CONFIGURATION.value],
            "integrity_verified": self.verify_integrity() if self.config.enable_hash_chain else None,
        }

    def verify_integrity(self) -> bool:
        """Recomputes every record's hash and checks each link to its predecessor. The chain must start
        at the first record ever written (previous hash None) unless older files were rotated out, and
        must end at the last hash this logger wrote (so a truncated tail is detected too)."""
        self.flush()
        prev, first = None, True
        for p in self._files():
            with open(p) as f:
                recs = [AuditEvent.from_dict(json.loads(ln)) for ln in f if ln.strip()]
            for e in recs:
                if e.hash is None or e.canonical_hash() != e.hash:
                    return False
                if first:
                    if p.endswith("audit_000000.log") and e.previous_hash is not None:
                        return False
                elif e.previous_hash != prev:
                    return False
                prev, first = e.hash, False
        return prev == self._last_hash
