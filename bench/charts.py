#!/usr/bin/env python3
"""SVG charts from bench JSONL (reference ``docs/make_charts.py``: SVG text
written directly, no graphics library).

    python bench/charts.py results.jsonl --x prompt_tokens --y decode_tok_s --out decode.svg
"""
from __future__ import annotations

import argparse
import json
import sys
from xml.sax.saxutils import escape


def line_chart(points: list[tuple[float, float]], title: str, xlabel: str, ylabel: str, w: int = 640,
               h: int = 360) -> str:
    pad = 56
    if not points:
        points = [(0.0, 0.0)]
    xs, ys = [p[0] for p in points], [p[1] for p in points]
    x0, x1 = min(xs), max(xs) if max(xs) > min(xs) else min(xs) + 1
    y0, y1 = 0.0, max(ys) * 1.1 if max(ys) > 0 else 1.0

    def px(x):
        return pad + (x - x0) / (x1 - x0) * (w - 2 * pad)

    def py(y):
        return h - pad - (y - y0) / (y1 - y0) * (h - 2 * pad)

    out = ['<svg xmlns="http://www.w3.org/2000/svg" width="%d" height="%d" font-family="sans-serif" '
           'font-size="12">' % (w, h),
           '<rect width="100%" height="100%" fill="white"/>',
           '<text x="%d" y="20" font-size="14">%s</text>' % (pad, escape(title)),
           '<line x1="%d" y1="%d" x2="%d" y2="%d" stroke="black"/>' % (pad, h - pad, w - pad, h - pad),
           '<line x1="%d" y1="%d" x2="%d" y2="%d" stroke="black"/>' % (pad, pad, pad, h - pad)]
    for i in range(5):
        yv = y0 + (y1 - y0) * i / 4
        out.append('<text x="4" y="%.1f">%.4g</text>' % (py(yv) + 4, yv))
        out.append('<line x1="%d" y1="%.1f" x2="%d" y2="%.1f" stroke="#ddd"/>' % (pad, py(yv), w - pad, py(yv)))
    pts = " ".join("%.1f,%.1f" % (px(x), py(y)) for x, y in sorted(points))
    out.append('<polyline fill="none" stroke="#1f77b4" stroke-width="2" points="%s"/>' % pts)
    for x, y in points:
        out.append('<circle cx="%.1f" cy="%.1f" r="3" fill="#1f77b4"/>' % (px(x), py(y)))
        out.append('<text x="%.1f" y="%.1f" font-size="10">%.4g</text>' % (px(x) + 4, py(y) - 6, y))
    out.append('<text x="%d" y="%d">%s</text>' % (w // 2 - 40, h - 12, escape(xlabel)))
    out.append('<text x="12" y="%d" transform="rotate(-90 12,%d)">%s</text>' % (h // 2, h // 2, escape(ylabel)))
    out.append("</svg>")
    return "\n".join(out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("jsonl")
    ap.add_argument("--x", required=True)
    ap.add_argument("--y", required=True)
    ap.add_argument("--title", default="")
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    pts = []
    for ln in open(a.jsonl):
        d = json.loads(ln)
        if d.get(a.x) is not None and d.get(a.y) is not None:
            pts.append((float(d[a.x]), float(d[a.y])))
    with open(a.out, "w") as f:
        f.write(line_chart(pts, a.title or "%s vs %s" % (a.y, a.x), a.x, a.y))
    return 0


if __name__ == "__main__":
    sys.exit(main())
