"""Terminal colour helpers: escape codes, environment rules, gradients."""
from scirs_b200.utils import colors as C


def test_codes_and_strip():
    s = C.colorize("x", C.Color.RED)
    assert s == "\x1b[31mx\x1b[0m" and C.strip_ansi(s) == "x"
    assert C.colorize_bg("y", C.Color.BRIGHT_BLUE) == "\x1b[104my\x1b[0m"
    assert C.stylize("z", C.Style.BOLD) == "\x1b[1mz\x1b[0m"
    assert C.colorize_and_style("w", C.Color.GREEN, style=C.Style.UNDERLINE) == "\x1b[32m\x1b[4mw\x1b[0m"
    assert C.colorize_and_style("plain") == "plain"


def test_supports_color_environment_rules():
    assert not C.supports_color({"TERM": "dumb", "FORCE_COLOR": "1"})
    assert not C.supports_color({"NO_COLOR": "1", "FORCE_COLOR": "1"})
    assert C.supports_color({"FORCE_COLOR": "1"})
    assert C.supports_color({"GITHUB_ACTIONS": "true"})

    class NotTty:
        def isatty(self):
            return False

    assert not C.supports_color({}, NotTty())


def test_gradients_cells_and_legends():
    on = C.ColorOptions(enabled=True, use_bright=False)
    assert [C.gradient_color(v, on) for v in (0.1, 0.6, 0.9)] == [C.Color.RED, C.Color.YELLOW, C.Color.GREEN]
    assert C.gradient_color(1.5, on) is None and C.gradient_color(0.5, C.ColorOptions(enabled=False)) is None
    bright = C.ColorOptions(enabled=True)
    assert [C.heatmap_gradient_color(v, bright) for v in (0.0, 0.3, 0.5, 0.7, 1.0)] == [
        C.Color.BRIGHT_BLUE, C.Color.BRIGHT_CYAN, C.Color.BRIGHT_YELLOW, C.Color.BRIGHT_RED, C.Color.BRIGHT_MAGENTA]
    assert C.strip_ansi(C.heatmap_cell(0.93, 0.93, bright)) == "0.93" and "\x1b[1m" in C.heatmap_cell(1, 0.9, bright)
    assert C.colored_metric_cell(3, 0.2, C.ColorOptions(enabled=False)) == "3"
    assert "Low (0.0-0.5)" in C.color_legend(on) and C.heatmap_color_legend(C.ColorOptions(enabled=False)) is None
    assert C.strip_ansi(C.heatmap_color_legend(on)).count("■") == 5
