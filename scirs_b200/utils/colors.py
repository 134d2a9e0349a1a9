"""Terminal colours for tables and reports (ANSI SGR escape sequences).

`supports_color()` follows the common conventions: TERM=dumb or a non-empty
NO_COLOR disables colour, a non-empty FORCE_COLOR or a CI runner enables it,
otherwise colour is used when the stream is a terminal. `gradient_color` maps
a score in [0, 1] to red (< 0.5) / yellow (< 0.7) / green, and
`heatmap_gradient_color` to blue / cyan / yellow / red / magenta in steps of
0.2; values outside [0, 1] get no colour.

Reference parity: scirs2-neural/src/utils/colors.rs:9-470 (Color, Style,
colorize / colorize_bg / stylize, supports_color, ColorOptions, gradient and
heat-map colours, coloured cells and legends).
"""
from __future__ import annotations

import dataclasses
import enum
import os
import sys

RESET = "\x1b[0m"


class Color(enum.Enum):
    BLACK = 30
    RED = 31
    GREEN = 32
    YELLOW = 33
    BLUE = 34
    MAGENTA = 35
    CYAN = 36
    WHITE = 37
    BRIGHT_BLACK = 90
    BRIGHT_RED = 91
    BRIGHT_GREEN = 92
    BRIGHT_YELLOW = 93
    BRIGHT_BLUE = 94
    BRIGHT_MAGENTA = 95
    BRIGHT_CYAN = 96
    BRIGHT_WHITE = 97

    @property
    def fg(self) -> str:
        return f"\x1b[{self.value}m"

    @property
    def bg(self) -> str:
        return f"\x1b[{self.value + 10}m"

    def bright(self, on: bool = True) -> "Color":
        if not on or self.value >= 90:
            return self
        return Color(self.value + 60)


class Style(enum.Enum):
    BOLD = 1
    DIM = 2
    ITALIC = 3
    UNDERLINE = 4
    BLINK = 5
    REVERSE = 7

    @property
    def code(self) -> str:
        return f"\x1b[{self.value}m"


def colorize(text, color: Color) -> str:
    return f"{color.fg}{text}{RESET}"


def colorize_bg(text, color: Color) -> str:
    return f"{color.bg}{text}{RESET}"


def stylize(text, style: Style) -> str:
    return f"{style.code}{text}{RESET}"


def colorize_and_style(text, color: Color | None = None, bg: Color | None = None, style: Style | None = None) -> str:
    pre = (color.fg if color else "") + (bg.bg if bg else "") + (style.code if style else "")
    return f"{pre}{text}{RESET}" if pre else str(text)


def supports_color(env=None, stream=None) -> bool:
    env = os.environ if env is None else env
    if env.get("TERM") == "dumb" or env.get("NO_COLOR"):
        return False
    if env.get("FORCE_COLOR") or "GITHUB_ACTIONS" in env or env.get("CI"):
        return True
    s = sys.stdout if stream is None else stream
    return bool(getattr(s, "isatty", lambda: False)())


@dataclasses.dataclass
class ColorOptions:
    enabled: bool = dataclasses.field(default_factory=supports_color)
    use_background: bool = True
    use_bright: bool = True


def gradient_color(value: float, options: ColorOptions) -> Color | None:
    if not options.enabled or not 0.0 <= value <= 1.0:
        return None
    c = Color.RED if value < 0.5 else Color.YELLOW if value < 0.7 else Color.GREEN
    return c.bright(options.use_bright)


_HEAT = (Color.BLUE, Color.CYAN, Color.YELLOW, Color.RED, Color.MAGENTA)


def heatmap_gradient_color(value: float, options: ColorOptions) -> Color | None:
    if not options.enabled or not 0.0 <= value <= 1.0:
        return None
    return _HEAT[min(4, int(value / 0.2))].bright(options.use_bright)


def colored_metric_cell(value, normalized: float, options: ColorOptions) -> str:
    c = gradient_color(normalized, options)
    return colorize(value, c) if c else str(value)


def heatmap_cell(value, normalized: float, options: ColorOptions) -> str:
    """Heat-map coloured text; values above 0.7 are also bold."""
    c = heatmap_gradient_color(normalized, options)
    if c is None:
        return str(value)
    return colorize(stylize(value, Style.BOLD) if normalized > 0.7 else value, c)


def color_legend(options: ColorOptions) -> str | None:
    if not options.enabled:
        return None
    parts = [(Color.RED, "Low (0.0-0.5)"), (Color.YELLOW, "Medium (0.5-0.7)"), (Color.GREEN, "High (0.7-1.0)")]
    return "Color Legend: " + " ".join(f"{colorize('■', c.bright(options.use_bright))} {t}" for c, t in parts)


def heatmap_color_legend(options: ColorOptions) -> str | None:
    if not options.enabled:
        return None
    names = ["Very Low (0.0-0.2)", "Low (0.2-0.4)", "Medium (0.4-0.6)", "High (0.6-0.8)", "Very High (0.8-1.0)"]
    return "Heatmap Legend: " + " ".join(f"{colorize('■', c.bright(options.use_bright))} {t}"
                                         for c, t in zip(_HEAT, names))


def strip_ansi(text: str) -> str:
    import re

    return re.sub(r"\x1b\[[0-9;]*m", "", text)
