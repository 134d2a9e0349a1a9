import io
import json

from scirs_b200.utils import logging as L


class Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t


def test_logger_levels_handlers_and_rate_limit(tmp_path):
    buf = io.StringIO()
    clk = Clock()
    rl = L.RateLimiter(L.RateLimitStrategy("sliding_window", max_events=2, window_s=10), clock=clk)
    log = L.Logger("train", L.LogLevel.INFO, [L.ConsoleLogHandler(buf, json_lines=True),
                                               L.FileLogHandler(str(tmp_path / "log.jsonl"))], rl)
    assert not log.debug("hidden")
    assert [log.info("step", loss=1.0) for _ in range(3)] == [True, True, False]
    assert log.error("boom")  # errors bypass the limiter
    clk.t = 11.0
    assert log.info("step")
    lines = [json.loads(x) for x in buf.getvalue().splitlines()]
    assert lines[0]["fields"] == {"loss": 1.0} and lines[2]["level"] == "ERROR"
    assert len((tmp_path / "log.jsonl").read_text().splitlines()) == 4
    assert rl.suppression_summary() == {"train:step": 1}
    tb = L.RateLimiter(L.RateLimitStrategy("token_bucket", capacity=2, refill_per_s=1.0), clock=clk)
    assert [tb.allow("k") for _ in range(3)] == [True, True, False]
    clk.t += 1.0
    assert tb.allow("k")
    fw = L.RateLimiter(L.RateLimitStrategy("fixed_window", max_events=1, window_s=5), clock=clk)
    assert fw.allow("a") and not fw.allow("a")
    clk.t += 5
    assert fw.allow("a")


def test_progress_tracker():
    clk = Clock()
    p = L.ProgressTracker("epoch", 100, update_interval_s=1.0, clock=clk)
    clk.t = 2.0
    st = p.update(50)
    assert st["percent"] == 50.0 and abs(st["eta_s"] - 2.0) < 1e-9
    clk.t = 2.5
    assert p.update(60) is None  # inside the update interval
    assert p.finish()["percent"] == 100.0
