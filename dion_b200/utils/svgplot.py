"""Dependency-free SVG charts (line, scatter, grouped and stacked bars).

The benchmark plots need only a handful of chart types; writing them as SVG
directly keeps the plotting tools usable on machines without matplotlib.

    fig = Figure(ncols=2, title="...")
    ax = fig.axes[0]
    ax.line(xs, ys, label="dion")
    ax.set(xlabel="step", ylabel="loss", logy=False)
    fig.save("out.svg")
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from html import escape
from typing import List, Optional, Sequence, Tuple

__all__ = ["Figure", "Axes", "PALETTE"]

PALETTE = ["#1f77b4", "#d62728", "#2ca02c", "#ff7f0e", "#9467bd", "#8c564b", "#e377c2", "#17becf", "#7f7f7f"]


def _nice_ticks(lo: float, hi: float, n: int = 5) -> List[float]:
    if not math.isfinite(lo) or not math.isfinite(hi):
        return []
    if hi <= lo:
        hi = lo + (abs(lo) or 1.0)
    raw = (hi - lo) / max(1, n)
    mag = 10 ** math.floor(math.log10(raw))
    step = min((s * mag for s in (1, 2, 2.5, 5, 10) if s * mag >= raw), default=10 * mag)
    t = math.ceil(lo / step) * step
    out = []
    while t <= hi + 1e-9 * step:
        out.append(round(t, 12))
        t += step
    return out


def _fmt(v: float) -> str:
    a = abs(v)
    if a != 0 and (a >= 1e5 or a < 1e-3):
        return f"{v:.2g}"
    if a >= 100 or float(v).is_integer():
        return f"{v:.0f}"
    return f"{v:.3g}"


@dataclass
class _Series:
    kind: str  # line | scatter | hline
    xs: List[float]
    ys: List[float]
    label: Optional[str]
    color: str
    dashed: bool = False
    markers: bool = False


@dataclass
class Axes:
    title: str = ""
    xlabel: str = ""
    ylabel: str = ""
    logy: bool = False
    series: List[_Series] = field(default_factory=list)
    bars: Optional[Tuple[List[str], List[str], List[List[float]], bool]] = None  # cats, groups, values, stacked
    _n: int = 0

    def _color(self, color: Optional[str]) -> str:
        if color:
            return color
        c = PALETTE[self._n % len(PALETTE)]
        self._n += 1
        return c

    def set(self, title: str = None, xlabel: str = None, ylabel: str = None, logy: bool = None) -> "Axes":
        if title is not None:
            self.title = title
        if xlabel is not None:
            self.xlabel = xlabel
        if ylabel is not None:
            self.ylabel = ylabel
        if logy is not None:
            self.logy = logy
        return self

    def line(self, xs: Sequence[float], ys: Sequence[float], label: str = None, color: str = None,
             dashed: bool = False, markers: bool = False) -> None:
        self.series.append(_Series("line", [float(x) for x in xs], [float(y) for y in ys], label, self._color(color),
                                   dashed, markers))

    def scatter(self, xs, ys, label: str = None, color: str = None) -> None:
        self.series.append(_Series("scatter", [float(x) for x in xs], [float(y) for y in ys], label,
                                   self._color(color)))

    def hline(self, y: float, label: str = None, color: str = "#888888") -> None:
        self.series.append(_Series("hline", [], [float(y)], label, color, dashed=True))

    def bar(self, categories: Sequence[str], groups: Sequence[str], values: Sequence[Sequence[float]],
            stacked: bool = False) -> None:
        """values[g][c]: value of group g (legend entry) for category c (x position)."""
        self.bars = ([str(c) for c in categories], [str(g) for g in groups],
                     [[float(v) for v in row] for row in values], stacked)

    # ------------------------------------------------------------ rendering
    def _render(self, x0: float, y0: float, w: float, h: float) -> List[str]:
        out: List[str] = []
        L, R, T, B = 64, 12, 28, 44
        px0, py0, pw, ph = x0 + L, y0 + T, w - L - R, h - T - B
        out.append(f'<text x="{x0 + w / 2:.1f}" y="{y0 + 18:.1f}" text-anchor="middle" font-size="14" '
                   f'font-weight="bold">{escape(self.title)}</text>')
        out.append(f'<rect x="{px0:.1f}" y="{py0:.1f}" width="{pw:.1f}" height="{ph:.1f}" fill="none" '
                   f'stroke="#444"/>')
        tf = (lambda v: math.log10(v) if v > 0 else float("nan")) if self.logy else (lambda v: v)
        legend: List[Tuple[str, str, bool]] = []
        if self.bars is not None:
            cats, groups, vals, stacked = self.bars
            tops = ([sum(vals[g][c] for g in range(len(groups))) for c in range(len(cats))] if stacked
                    else [max(vals[g][c] for g in range(len(groups))) for c in range(len(cats))])
            ymax = max(tops + [0.0]) * 1.08 or 1.0
            ticks = _nice_ticks(0.0, ymax)
            sy = lambda v: py0 + ph - v / ymax * ph  # noqa: E731
            for t in ticks:
                out.append(f'<line x1="{px0}" x2="{px0 + pw}" y1="{sy(t):.1f}" y2="{sy(t):.1f}" stroke="#ddd"/>')
                out.append(f'<text x="{px0 - 4}" y="{sy(t) + 4:.1f}" text-anchor="end" font-size="10">{_fmt(t)}</text>')
            slot = pw / max(1, len(cats))
            colors = [PALETTE[i % len(PALETTE)] for i in range(len(groups))]
            for c, cat in enumerate(cats):
                base = 0.0
                for g in range(len(groups)):
                    v = vals[g][c]
                    if stacked:
                        bx, bw = px0 + c * slot + slot * 0.15, slot * 0.7
                        y_top, y_bot = sy(base + v), sy(base)
                        base += v
                    else:
                        bw = slot * 0.8 / max(1, len(groups))
                        bx = px0 + c * slot + slot * 0.1 + g * bw
                        y_top, y_bot = sy(v), sy(0.0)
                    out.append(f'<rect x="{bx:.1f}" y="{y_top:.1f}" width="{bw:.1f}" height="{max(0.0, y_bot - y_top):.1f}" '
                               f'fill="{colors[g]}"/>')
                out.append(f'<text x="{px0 + (c + 0.5) * slot:.1f}" y="{py0 + ph + 14:.1f}" text-anchor="middle" '
                           f'font-size="10">{escape(cat)}</text>')
            legend = [(g, colors[i], False) for i, g in enumerate(groups)]
        else:
            xs = [x for s in self.series if s.kind != "hline" for x in s.xs if math.isfinite(x)]
            ys = [tf(y) for s in self.series for y in s.ys]
            ys = [y for y in ys if math.isfinite(y)]
            if not xs:
                xs = [0.0, 1.0]
            if not ys:
                ys = [0.0, 1.0]
            xlo, xhi = min(xs), max(xs)
            ylo, yhi = min(ys), max(ys)
            if xhi == xlo:
                xhi = xlo + 1
            pad = (yhi - ylo) * 0.05 or (abs(yhi) * 0.05 or 1.0)
            ylo, yhi = ylo - pad, yhi + pad
            sx = lambda v: px0 + (v - xlo) / (xhi - xlo) * pw  # noqa: E731
            sy = lambda v: py0 + ph - (tf(v) - ylo) / (yhi - ylo) * ph  # noqa: E731
            for t in _nice_ticks(xlo, xhi):
                out.append(f'<text x="{sx(t):.1f}" y="{py0 + ph + 14:.1f}" text-anchor="middle" font-size="10">'
                           f'{_fmt(t)}</text>')
            for t in _nice_ticks(ylo, yhi):
                yy = py0 + ph - (t - ylo) / (yhi - ylo) * ph
                lab = _fmt(10 ** t) if self.logy else _fmt(t)
                out.append(f'<line x1="{px0}" x2="{px0 + pw}" y1="{yy:.1f}" y2="{yy:.1f}" stroke="#eee"/>')
                out.append(f'<text x="{px0 - 4}" y="{yy + 4:.1f}" text-anchor="end" font-size="10">{lab}</text>')
            for s in self.series:
                dash = ' stroke-dasharray="5,4"' if s.dashed else ""
                if s.kind == "hline":
                    yy = sy(s.ys[0])
                    out.append(f'<line x1="{px0}" x2="{px0 + pw}" y1="{yy:.1f}" y2="{yy:.1f}" stroke="{s.color}"{dash}/>')
                else:
                    pts = [(sx(x), sy(y)) for x, y in zip(s.xs, s.ys) if math.isfinite(tf(y))]
                    if s.kind == "line" and len(pts) > 1:
                        path = " ".join(f"{x:.1f},{y:.1f}" for x, y in pts)
                        out.append(f'<polyline points="{path}" fill="none" stroke="{s.color}" stroke-width="1.8"{dash}/>')
                    if s.kind == "scatter" or s.markers or len(pts) == 1:
                        out.extend(f'<circle cx="{x:.1f}" cy="{y:.1f}" r="3" fill="{s.color}"/>' for x, y in pts)
                if s.label:
                    legend.append((s.label, s.color, s.dashed))
        out.append(f'<text x="{px0 + pw / 2:.1f}" y="{y0 + h - 8:.1f}" text-anchor="middle" font-size="12">'
                   f'{escape(self.xlabel)}</text>')
        out.append(f'<text transform="translate({x0 + 14:.1f},{py0 + ph / 2:.1f}) rotate(-90)" text-anchor="middle" '
                   f'font-size="12">{escape(self.ylabel)}</text>')
        for i, (lab, col, dashed) in enumerate(legend):
            ly = py0 + 12 + 14 * i
            dash = ' stroke-dasharray="4,3"' if dashed else ""
            out.append(f'<line x1="{px0 + pw - 120}" x2="{px0 + pw - 100}" y1="{ly - 4}" y2="{ly - 4}" '
                       f'stroke="{col}" stroke-width="3"{dash}/>')
            out.append(f'<text x="{px0 + pw - 96}" y="{ly:.1f}" font-size="10">{escape(lab)}</text>')
        return out


class Figure:
    def __init__(self, ncols: int = 1, nrows: int = 1, width: int = 520, height: int = 360, title: str = ""):
        self.ncols, self.nrows, self.w, self.h, self.title = ncols, nrows, width, height, title
        self.axes = [Axes() for _ in range(ncols * nrows)]

    def to_svg(self) -> str:
        top = 24 if self.title else 0
        W, H = self.ncols * self.w, self.nrows * self.h + top
        parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" viewBox="0 0 {W} {H}" '
                 f'font-family="sans-serif">', f'<rect width="{W}" height="{H}" fill="white"/>']
        if self.title:
            parts.append(f'<text x="{W / 2:.1f}" y="18" text-anchor="middle" font-size="15" font-weight="bold">'
                         f'{escape(self.title)}</text>')
        for i, ax in enumerate(self.axes):
            r, c = divmod(i, self.ncols)
            parts.extend(ax._render(c * self.w, top + r * self.h, self.w, self.h))
        parts.append("</svg>")
        return "\n".join(parts)

    def save(self, path: str) -> str:
        with open(path, "w") as f:
            f.write(self.to_svg())
        return path
