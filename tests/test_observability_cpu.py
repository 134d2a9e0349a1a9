"""Tracing (span trees, W3C header round trips, samplers, exporters) and the
hash-chained audit log (tamper detection, rotation, search, alerts)."""
import json
from datetime import timedelta

import pytest

from scirs_b200.utils import observability as O


def test_traceparent_and_baggage_round_trip():
    ctx = O.TraceContext().with_baggage("user", "a b,c").with_baggage("tenant", "x=1").with_tracestate("k=v")
    tp = ctx.to_traceparent()
    assert tp.startswith("00-") and len(tp) == 55 and tp.endswith("-01")
    remote = O.TraceContext.from_headers(ctx.headers())
    assert remote.trace_id == ctx.trace_id and remote.parent_span_id == ctx.span_id
    assert remote.span_id != ctx.span_id and remote.is_remote and remote.is_sampled
    assert remote.baggage == {"user": "a b,c", "tenant": "x=1"} and remote.tracestate == "k=v"
    for bad in ("01-" + tp[3:], "00-" + "0" * 32 + tp[35:], "00-abc-def-01", tp.upper(), "garbage"):
        with pytest.raises(ValueError):
            O.TraceContext.from_traceparent(bad)
    assert O.TraceContext().with_baggage_header("a=1;prop=2, b = %20x").baggage == {"a": "1", "b": " x"}


def test_span_tree_attributes_events_and_errors():
    exp = O.InMemoryExporter()
    tr = O.TracingSystem(O.TracingConfig(service_name="svc", default_attributes={"rank": 0}), exp)
    with tr.start_span("step", attributes={"step": 3}) as root:
        root.add_event("loaded", {"n": 2}).add_metric("tokens", 1024)
        with tr.start_span("forward") as fwd:
            assert tr.current_span() is fwd
            with tr.start_span("attention"):
                pass
        with pytest.raises(ZeroDivisionError):
            with tr.start_span("bad"):
                1 / 0
    assert tr.current_span() is None
    tr.flush()
    spans = {s.name: s for s in exp.spans}
    assert set(spans) == {"step", "forward", "attention", "bad"}
    assert len({s.context.trace_id for s in exp.spans}) == 1
    assert spans["forward"].context.parent_span_id == spans["step"].context.span_id
    assert spans["attention"].context.parent_span_id == spans["forward"].context.span_id
    assert spans["step"].context.parent_span_id is None
    assert spans["bad"].status == O.SpanStatus.ERROR and "ZeroDivisionError" in spans["bad"].error
    assert spans["step"].status == O.SpanStatus.OK
    s = spans["step"]
    assert s.attributes["step"] == 3 and s.attributes["rank"] == 0 and s.attributes["service.name"] == "svc"
    assert s.metrics["tokens"] == 1024 and s.events[0].name == "loaded"
    assert s.duration_ns >= spans["forward"].duration_ns >= 0
    m = tr.get_metrics()
    assert m.spans_started == m.spans_finished == m.spans_exported == 4 and m.active_spans == 0


def test_remote_parent_continues_trace():
    exp = O.InMemoryExporter()
    tr = O.TracingSystem(exporter=exp)
    caller = O.TraceContext()
    with tr.start_span("handle", kind=O.SpanKind.SERVER, parent=O.TraceContext.from_traceparent(
            caller.to_traceparent())):
        pass
    with tr.start_span("local_child", parent=caller):
        pass
    tr.flush()
    a, b = exp.spans
    assert a.context.trace_id == b.context.trace_id == caller.trace_id
    assert a.context.parent_span_id == b.context.parent_span_id == caller.span_id
    assert a.kind == O.SpanKind.SERVER


def test_in_span_and_decorator():
    exp = O.InMemoryExporter()
    tr = O.init_tracing(exporter=exp)
    assert O.global_tracer() is tr

    @O.traced("work")
    def work(x):
        return O.global_tracer().current_span().span.name, x + 1

    assert work(1) == ("work", 2)
    sp = tr.start_span("outer")
    assert sp.in_span(lambda: tr.current_span()) is sp
    with pytest.raises(KeyError):
        sp.in_span(lambda: {}["k"])
    sp.end()
    sp.end()  # idempotent
    tr.flush()
    assert [s.name for s in exp.spans] == ["work", "outer"] and exp.spans[1].status == O.SpanStatus.ERROR


def test_samplers():
    always, never = O.ProbabilitySampler(1.0), O.ProbabilitySampler(0.0)
    ctxs = [O.TraceContext() for _ in range(2000)]
    assert all(always.should_sample(c) for c in ctxs) and not any(never.should_sample(c) for c in ctxs)
    half = sum(O.ProbabilitySampler(0.5).should_sample(c) for c in ctxs)
    assert 850 < half < 1150
    c0 = ctxs[0]
    assert len({O.ProbabilitySampler(0.3).should_sample(c0) for _ in range(10)}) == 1  # decided by the id
    t = [0.0]
    rl = O.RateLimitingSampler(10, clock=lambda: t[0])
    assert sum(rl.should_sample(c) for c in ctxs[:50]) == 10
    t[0] += 0.5
    assert sum(rl.should_sample(c) for c in ctxs[:50]) == 5
    ad = O.AdaptiveSampler(1.0, target_per_second=100, clock=lambda: t[0])
    for k in range(3):
        for c in ctxs[:1000]:
            ad.should_sample(c)
        t[0] += 1.0
    ad.should_sample(ctxs[0])
    seen, sampled, rate = ad.get_stats()
    assert seen == 3001 and abs(rate - 0.1) < 1e-9 and sampled < seen


def test_unsampled_traces_are_not_exported_and_children_follow():
    exp = O.InMemoryExporter()
    tr = O.TracingSystem(exporter=exp, sampler=O.ProbabilitySampler(0.0))
    with tr.start_span("root"):
        with tr.start_span("child") as c:
            assert not c.context.is_sampled
    tr.flush()
    assert exp.spans == [] and tr.get_metrics().spans_not_sampled == 2


def test_max_active_spans_and_timeouts():
    exp = O.InMemoryExporter()
    tr = O.TracingSystem(O.TracingConfig(max_active_spans=2, span_timeout_s=0.0), exp)
    a, b, c = tr.start_span("a"), tr.start_span("b"), tr.start_span("c")
    assert tr.get_metrics().spans_dropped == 1
    assert tr.cleanup_expired_spans() == 2
    c.end()
    tr.flush()
    assert sorted(s.name for s in exp.spans) == ["a", "b"]
    assert all(s.error == "span timed out" for s in exp.spans)


def test_exporters(tmp_path):
    inner = O.InMemoryExporter()
    batch = O.BatchExporter(inner, batch_size=3)
    chrome = O.ChromeTraceExporter(str(tmp_path / "trace.json"), rank=3)
    jl = tmp_path / "spans.jsonl"
    for exp in (batch, chrome, O.JsonlExporter(str(jl))):
        tr = O.TracingSystem(O.TracingConfig(export_batch_size=1000), exp)
        for i in range(7):
            with tr.start_span(f"s{i}") as s:
                s.add_event("e")
        tr.flush()
    assert len(inner.spans) == 7 and batch.batches_sent == 3
    doc = json.load(open(chrome.write()))
    xs = [e for e in doc["traceEvents"] if e["ph"] == "X"]
    assert len(xs) == 7 and all(e["pid"] == 3 and e["dur"] >= 0 for e in xs)
    rows = [json.loads(x) for x in jl.read_text().splitlines()]
    assert [r["name"] for r in rows] == [f"s{i}" for i in range(7)] and rows[0]["events"][0]["name"] == "e"


def test_resource_attribution_merge():
    a = O.ResourceAttribution(cpu_time_ns=5, memory_bytes=100, io_operations=1, gpu_memory_bytes=7)
    a.merge(O.ResourceAttribution(cpu_time_ns=3, memory_bytes=50, io_operations=2, gpu_memory_bytes=9))
    assert (a.cpu_time_ns, a.memory_bytes, a.io_operations, a.gpu_memory_bytes) == (8, 100, 3, 9)


# ---------------------------------------------------------------------------- audit


def _logger(tmp_path, **kw):
    return O.AuditLogger(O.AuditConfig(log_directory=str(tmp_path / "audit"), buffer_size=4, **kw))


def test_audit_log_chain_search_and_stats(tmp_path):
    log = _logger(tmp_path)
    log.log_authentication("alice", True, source_ip="10.0.0.1")
    log.log_authentication("mallory", False)
    log.log_data_access("alice", "dataset/train", "read")
    log.log_configuration_change("bob", "lr", 0.1, 0.01)
    log.log_security_event("port_scan", O.EventSeverity.CRITICAL, "blocked", user_id="mallory")
    ev = (O.AuditEventBuilder(O.EventCategory.COMPLIANCE, "export").user_id("carol").compliance_tag("gdpr")
          .data_classification(O.DataClassification.CONFIDENTIAL).correlation_id("job-7").metadata("rows", 10).build())
    log.log_event(ev)
    assert log.verify_integrity()
    all_ev = log.search_events()
    assert len(all_ev) == 6 and all_ev[0].previous_hash is None
    assert all(b.previous_hash == a.hash for a, b in zip(all_ev, all_ev[1:]))
    assert [e.action for e in log.search_events(user_id="alice")] == ["login", "read"]
    assert len(log.search_events(category=O.EventCategory.AUTHENTICATION)) == 2
    assert log.search_events(action="config")[0].metadata == {"old_value": 0.1, "new_value": 0.01}
    assert len(log.search_events(limit=2)) == 2
    assert log.search_events(start=O._now() + timedelta(hours=1)) == []
    got = log.search_events(category=O.EventCategory.COMPLIANCE)[0]
    assert got.data_classification == O.DataClassification.CONFIDENTIAL and got.compliance_tags == ["gdpr"]
    st = log.get_statistics(1)
    assert st["total_events"] == 6 and st["unique_users"] == 4 and st["by_outcome"]["failure"] == 1
    rep = log.export_compliance_report(O._now() - timedelta(days=1), O._now() + timedelta(days=1))
    assert rep["failed_authentications"] == 1 and rep["configuration_changes"] == 1 and rep["integrity_verified"]


def _files(log):
    return log._files()


def test_audit_tamper_detection(tmp_path):
    log = _logger(tmp_path)
    for i in range(5):
        log.log_data_access("u", f"r{i}", "read")
    log.flush()
    p = _files(log)[0]
    lines = open(p).read().splitlines()

    def check(new_lines):
        open(p, "w").write("\n".join(new_lines) + "\n")
        ok = log.verify_integrity()
        open(p, "w").write("\n".join(lines) + "\n")
        return ok

    assert check(lines)
    edited = json.loads(lines[2])
    edited["resource_id"] = "evil"
    assert not check(lines[:2] + [json.dumps(edited)] + lines[3:])  # edited record
    assert not check(lines[:2] + lines[3:])  # deleted middle record
    assert not check(lines[1:])  # deleted first record
    assert not check(lines[:-1])  # truncated tail
    assert not check([lines[1], lines[0]] + lines[2:])  # reordered


def test_audit_rotation_and_reopen(tmp_path):
    log = _logger(tmp_path, max_file_size=600, max_files=50)
    for i in range(12):
        log.log_data_access("u", f"r{i}", "read")
    log.flush()
    assert len(_files(log)) > 1 and log.verify_integrity()
    again = _logger(tmp_path, max_file_size=600, max_files=50)  # continues the chain from the files
    again.log_data_access("u", "later", "read")
    assert again.verify_integrity() and len(again.search_events()) == 13
    capped = _logger(tmp_path, max_file_size=600, max_files=2)
    capped.log_data_access("u", "x", "read")
    capped.flush()
    assert len(_files(capped)) == 2 and capped.verify_integrity()  # older files rotated out


def test_alert_manager_thresholds_and_cooldown(tmp_path):
    t = [0.0]
    am = O.AlertManager(O.AlertingConfig(failed_auth_threshold=3, window_s=10, cooldown_s=100), clock=lambda: t[0])
    fired = []
    am.add_handler(lambda k, e: fired.append(k))
    fail = O.AuditEventBuilder(O.EventCategory.AUTHENTICATION, "login").outcome(O.EventOutcome.FAILURE).build()
    assert [am.process_event(fail) for _ in range(3)] == [False, False, True]
    assert not am.process_event(fail)  # cooldown
    t[0] = 200.0
    assert not am.process_event(fail)  # the window forgot the old failures
    assert am.process_event(O.AuditEventBuilder(O.EventCategory.SECURITY, "x").severity(
        O.EventSeverity.CRITICAL).build())
    assert fired == ["failed_authentication", "critical_event"]
    log = _logger(tmp_path, alerting=O.AlertingConfig(failed_auth_threshold=2))
    got = []
    log.alerts.add_handler(lambda k, e: got.append((k, e.user_id)))
    log.log_authentication("m", False)
    log.log_authentication("m", False)
    assert got == [("failed_authentication", "m")]


def test_otlp_json_exporter(tmp_path):
    p = tmp_path / "otlp.jsonl"
    exp = O.OtlpJsonExporter(str(p), "trainer", {"rank": 3})
    tr = O.TracingSystem(exporter=exp)
    with tr.start_span("step", kind=O.SpanKind.SERVER, attributes={"step": 7, "lr": 0.1, "ok": True}) as s:
        s.add_metric("tokens", 2048).add_event("ckpt", {"path": "x"})
        with tr.start_span("fwd"):
            pass
    tr.flush()
    doc = json.loads(p.read_text().splitlines()[0])
    rs = doc["resourceSpans"][0]
    assert {"key": "service.name", "value": {"stringValue": "trainer"}} in rs["resource"]["attributes"]
    assert {"key": "rank", "value": {"intValue": "3"}} in rs["resource"]["attributes"]
    spans = {x["name"]: x for x in rs["scopeSpans"][0]["spans"]}
    st, fwd = spans["step"], spans["fwd"]
    assert len(st["traceId"]) == 32 and len(st["spanId"]) == 16 and "parentSpanId" not in st
    assert fwd["parentSpanId"] == st["spanId"] and fwd["traceId"] == st["traceId"]
    assert st["kind"] == 2 and st["status"] == {"code": 1}
    assert int(st["endTimeUnixNano"]) >= int(st["startTimeUnixNano"])
    attrs = {a["key"]: a["value"] for a in st["attributes"]}
    assert attrs["step"] == {"intValue": "7"} and attrs["lr"] == {"doubleValue": 0.1}
    assert attrs["ok"] == {"boolValue": True} and attrs["metric.tokens"] == {"doubleValue": 2048.0}
    assert st["events"][0]["name"] == "ckpt"
