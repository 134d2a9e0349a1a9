import time

from scirs_b200.utils.profiling import Profiler, SystemMonitor


def test_nested_sections_flame_graph(tmp_path):
    p = Profiler()
    with p.section("step"):
        with p.section("forward"):
            time.sleep(0.01)
        with p.section("backward"):
            time.sleep(0.02)
    folded = dict(line.rsplit(" ", 1) for line in p.folded().splitlines())
    assert set(folded) == {"step", "step;forward", "step;backward"}
    assert int(folded["step;backward"]) > int(folded["step;forward"]) > 0
    svg = p.flame_graph_svg(str(tmp_path / "f.svg"))
    assert svg.startswith("<svg") and "backward" in svg and (tmp_path / "f.svg").exists()
    assert p.calls["step"] == 1 and "forward" in p.report()


def test_system_monitor():
    m = SystemMonitor(interval=0.01).start()
    time.sleep(0.05)
    samples = m.stop()
    assert samples and samples[0]["rss_bytes"] > 0 and "cpu_percent" in samples[0]
