"""Headless visualisation: files and text, no display or graphics stack.

  ascii_plot(values)              text line chart of a series (loss curves)
  svg_line_plot(series, path)     SVG file with one polyline per series
  heatmap_svg(matrix, path)       SVG heat map (attention weights, feature maps)
  ActivationVisualizer(model)     forward hooks that cache each layer's
                                  output; per-layer statistics, histograms and
                                  channel-aggregated feature maps
  attention_maps(weights)         per-head / averaged attention matrices
  network_summary(model)          layer table: name, type, parameters, output shape
  training_curves_svg(history)    train / validation curves of a History

Reference parity: scirs2-neural/src/visualization/{activations.rs:20-230,
attention.rs:18-210, network.rs, training.rs} (SVG / ASCII output).
"""
from __future__ import annotations

import html
import math

import torch
import torch.nn as nn


def ascii_plot(values, width: int = 60, height: int = 12, title: str = "") -> str:
    vals = [float(v) for v in values]
    if not vals:
        return title
    lo, hi = min(vals), max(vals)
    span = hi - lo or 1.0
    cols = [vals[min(len(vals) - 1, int(i * len(vals) / width))] for i in range(width)]
    grid = [[" "] * width for _ in range(height)]
    for x, v in enumerate(cols):
        y = height - 1 - int(round((v - lo) / span * (height - 1)))
        grid[y][x] = "*"
    lines = [title] if title else []
    for r, row in enumerate(grid):
        label = hi - span * r / (height - 1)
        lines.append(f"{label:>10.4g} |" + "".join(row))
    lines.append(" " * 11 + "+" + "-" * width)
    return "\n".join(lines)


_COLORS = ["#1f77b4", "#d62728", "#2ca02c", "#ff7f0e", "#9467bd", "#8c564b"]


def svg_line_plot(series: dict, path: str, title: str = "", width: int = 640, height: int = 360) -> str:
    pad = 40
    allv = [float(v) for s in series.values() for v in s] or [0.0]
    lo, hi = min(allv), max(allv)
    span = hi - lo or 1.0
    n = max((len(s) for s in series.values()), default=1)
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}">',
             f'<rect width="{width}" height="{height}" fill="white"/>',
             f'<text x="{width / 2}" y="20" text-anchor="middle" font-size="14">{html.escape(title)}</text>',
             f'<line x1="{pad}" y1="{height - pad}" x2="{width - pad}" y2="{height - pad}" stroke="black"/>',
             f'<line x1="{pad}" y1="{pad}" x2="{pad}" y2="{height - pad}" stroke="black"/>',
             f'<text x="4" y="{pad}" font-size="10">{hi:.4g}</text>',
             f'<text x="4" y="{height - pad}" font-size="10">{lo:.4g}</text>']
    for k, (name, s) in enumerate(series.items()):
        pts = " ".join(f"{pad + (width - 2 * pad) * i / max(n - 1, 1):.1f},"
                       f"{height - pad - (height - 2 * pad) * (float(v) - lo) / span:.1f}" for i, v in enumerate(s))
        c = _COLORS[k % len(_COLORS)]
        parts.append(f'<polyline fill="none" stroke="{c}" stroke-width="1.5" points="{pts}"/>')
        parts.append(f'<text x="{width - pad - 100}" y="{pad + 14 * k}" font-size="11" fill="{c}">'
                     f'{html.escape(str(name))}</text>')
    parts.append("</svg>")
    svg = "\n".join(parts)
    with open(path, "w") as f:
        f.write(svg)
    return svg


def _viridis_like(t: float) -> str:
    t = min(max(t, 0.0), 1.0)
    r, g, b = int(68 + t * (253 - 68)), int(1 + t * (231 - 1)), int(84 + (1 - 2 * abs(t - 0.5)) * 60)
    return f"rgb({r},{g},{b})"


def heatmap_svg(matrix, path: str, title: str = "", cell: int = 8, row_labels=None, col_labels=None) -> str:
    m = torch.as_tensor(matrix, dtype=torch.float32).cpu()
    lo, hi = float(m.min()), float(m.max())
    span = hi - lo or 1.0
    R, C = m.shape
    off = 30 if (row_labels or col_labels) else 0
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{C * cell + off + 10}" height="{R * cell + off + 30}">',
             f'<text x="4" y="14" font-size="12">{html.escape(title)}</text>']
    for i in range(R):
        for j in range(C):
            parts.append(f'<rect x="{off + j * cell}" y="{off + 20 + i * cell}" width="{cell}" height="{cell}" '
                         f'fill="{_viridis_like((float(m[i, j]) - lo) / span)}"/>')
    parts.append("</svg>")
    svg = "\n".join(parts)
    with open(path, "w") as f:
        f.write(svg)
    return svg


class ActivationVisualizer:
    """Caches the outputs of the chosen layers (all leaf modules by default)
    on each forward pass."""

    def __init__(self, model: nn.Module, layers: list[str] | None = None):
        self.cache: dict[str, torch.Tensor] = {}
        self._hooks = []
        for name, mod in model.named_modules():
            if (layers is None and len(list(mod.children())) == 0 and name) or (layers and name in layers):
                self._hooks.append(mod.register_forward_hook(self._hook(name)))

    def _hook(self, name):
        def fn(mod, inp, out):
            if isinstance(out, torch.Tensor):
                self.cache[name] = out.detach()
        return fn

    def get_cached_activations(self, name: str):
        return self.cache.get(name)

    def clear_cache(self):
        self.cache.clear()

    def statistics(self) -> dict:
        out = {}
        for k, v in self.cache.items():
            f = v.float()
            out[k] = {"mean": float(f.mean()), "std": float(f.std()) if f.numel() > 1 else 0.0,
                      "min": float(f.min()), "max": float(f.max()),
                      "sparsity": float((f == 0).float().mean()), "shape": tuple(v.shape)}
        return out

    def histogram(self, name: str, bins: int = 32):
        f = self.cache[name].float().flatten().cpu()
        counts = torch.histc(f, bins=bins, min=float(f.min()), max=float(f.max()))
        edges = torch.linspace(float(f.min()), float(f.max()), bins + 1)
        return counts, edges

    def feature_map(self, name: str, sample: int = 0, aggregation: str = "mean") -> torch.Tensor:
        """[C, H, W] activations of one sample reduced over channels."""
        x = self.cache[name][sample].float()
        return {"mean": x.mean(0), "max": x.amax(0), "sum": x.sum(0)}[aggregation]

    def remove(self):
        for h in self._hooks:
            h.remove()


def attention_maps(weights: torch.Tensor, heads="all", aggregation: str = "mean") -> torch.Tensor:
    """weights [B?, H, S, S] -> one [S, S] map: head `heads` (int) or the
    mean / max over heads."""
    w = weights.float()
    if w.dim() == 4:
        w = w[0]
    if isinstance(heads, int):
        return w[heads]
    return w.mean(0) if aggregation == "mean" else w.amax(0)


def network_summary(model: nn.Module, example_input: torch.Tensor | None = None) -> str:
    shapes: dict[str, tuple] = {}
    hooks = []
    if example_input is not None:
        for name, mod in model.named_modules():
            if name and len(list(mod.children())) == 0:
                hooks.append(mod.register_forward_hook(
                    lambda m, i, o, n=name: shapes.__setitem__(n, tuple(o.shape) if isinstance(o, torch.Tensor) else ())))
        with torch.no_grad():
            model(example_input)
        for h in hooks:
            h.remove()
    rows = [("layer", "type", "params", "output")]
    total = 0
    for name, mod in model.named_modules():
        if not name or list(mod.children()):
            continue
        n = sum(p.numel() for p in mod.parameters(recurse=False))
        total += n
        rows.append((name, type(mod).__name__, f"{n:,}", str(shapes.get(name, ""))))
    w = [max(len(r[i]) for r in rows) for i in range(4)]
    lines = ["  ".join(r[i].ljust(w[i]) for i in range(4)) for r in rows]
    lines.insert(1, "-" * len(lines[0]))
    lines.append(f"total parameters: {total:,}")
    return "\n".join(lines)


def training_curves_svg(history, path: str, title: str = "training") -> str:
    """`history`: a dict of metric -> list, or an object with such a dict in
    `.history`."""
    series = history if isinstance(history, dict) else getattr(history, "history", {})
    series = {k: v for k, v in series.items() if v and all(isinstance(x, (int, float)) and math.isfinite(x) for x in v)}
    return svg_line_plot(series, path, title)
