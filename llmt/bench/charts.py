"""SVG charts of ladder / profile / scaling-model results (reference: make_charts.py and the
scaling model's plots, which need matplotlib; this writes plain SVG so it runs anywhere). The
architecture label comes from the result file's env info, never a hard-coded name.

    python -m llmt.bench.charts results/ladder_small.json --out results/ladder_small.svg
    python -m llmt.perf.scaling --gpus 8,16,32,64,128,256,512,1024 --json s.json
    python -m llmt.bench.charts s.json --out scaling.svg      # MFU vs GPUs per model
"""
from __future__ import annotations

import argparse
import html
import json


def bar_svg(labels, values, title, unit, width=900, bar_h=22):
    h = 60 + bar_h * len(labels)
    vmax = max(values) if values else 1.0
    x0, x1 = 330, width - 90
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{h}" font-family="sans-serif" font-size="12">',
           f'<text x="10" y="22" font-size="15">{html.escape(title)}</text>']
    for i, (lab, v) in enumerate(zip(labels, values)):
        y = 40 + i * bar_h
        w = (x1 - x0) * (v / vmax if vmax else 0)
        color = "#3b7dd8" if "native" in lab.lower() or lab.startswith("N") else "#9aa5b1"
        out.append(f'<text x="{x0 - 6}" y="{y + 15}" text-anchor="end">{html.escape(lab[:52])}</text>')
        out.append(f'<rect x="{x0}" y="{y + 3}" width="{w:.1f}" height="{bar_h - 6}" fill="{color}"/>')
        out.append(f'<text x="{x0 + w + 4:.1f}" y="{y + 15}">{v:,.0f} {html.escape(unit)}</text>')
    out.append("</svg>")
    return "\n".join(out)


def ladder_chart(res):
    rows = [r for r in res["rows"] if r.get("status") == "ok"]
    title = f"training tokens/s, {res.get('size')} b{res.get('batch')} s{res.get('seq')} ({res.get('arch', '?')})"
    return bar_svg([r["name"] for r in rows], [r["tokens_per_s"] for r in rows], title, "tok/s")


def profile_chart(res):
    b = res["buckets_pct"]
    return bar_svg(list(b), list(b.values()), f"GPU time buckets ({res['config']})", "%")


def line_svg(series, title, xlabel, ylabel, width=900, height=420):
    """series: {name: [(x, y), ...]} on a log2 x axis and a linear y axis from 0."""
    pts = [p for s in series.values() for p in s]
    if not pts:
        return f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="40"><text y="20">no data</text></svg>'
    import math
    xs = [math.log2(x) for x, _ in pts]
    xlo, xhi = min(xs), max(xs) if max(xs) > min(xs) else min(xs) + 1
    yhi = max(y for _, y in pts) * 1.1 or 1.0
    L, R, T, B = 70, width - 180, 40, height - 50

    def px(x):
        return L + (R - L) * (math.log2(x) - xlo) / (xhi - xlo)

    def py(y):
        return B - (B - T) * y / yhi

    colors = ["#3b7dd8", "#e8684a", "#5ab06e", "#9a6fd1", "#f0b429", "#6b7280"]
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" font-family="sans-serif" '
           f'font-size="12">', f'<text x="10" y="22" font-size="15">{html.escape(title)}</text>',
           f'<line x1="{L}" y1="{B}" x2="{R}" y2="{B}" stroke="#333"/>',
           f'<line x1="{L}" y1="{T}" x2="{L}" y2="{B}" stroke="#333"/>',
           f'<text x="{(L + R) / 2}" y="{height - 12}" text-anchor="middle">{html.escape(xlabel)}</text>',
           f'<text x="14" y="{(T + B) / 2}" transform="rotate(-90 14 {(T + B) / 2})" text-anchor="middle">'
           f'{html.escape(ylabel)}</text>']
    for x in sorted({x for x, _ in pts}):
        out.append(f'<text x="{px(x):.1f}" y="{B + 16}" text-anchor="middle">{x}</text>')
    for k in range(5):
        y = yhi * k / 4
        out.append(f'<text x="{L - 6}" y="{py(y) + 4:.1f}" text-anchor="end">{y:.3g}</text>')
    for i, (name, s) in enumerate(series.items()):
        c = colors[i % len(colors)]
        s = sorted(s)
        out.append('<polyline fill="none" stroke="{}" stroke-width="2" points="{}"/>'.format(
            c, " ".join(f"{px(x):.1f},{py(y):.1f}" for x, y in s)))
        for x, y in s:
            out.append(f'<circle cx="{px(x):.1f}" cy="{py(y):.1f}" r="3" fill="{c}"/>')
        out.append(f'<text x="{R + 12}" y="{T + 16 * i + 8}" fill="{c}">{html.escape(name)}</text>')
    out.append("</svg>")
    return "\n".join(out)


def scaling_chart(rows):
    """MFU (%) of the best layout per GPU count, one line per model (llmt.perf.scaling --json)."""
    series = {}
    best = {}
    for r in rows:
        key = (r["model"], r["gpus"])
        if key not in best or r["tokens_per_s"] > best[key]["tokens_per_s"]:
            best[key] = r
    for (model, n), r in best.items():
        series.setdefault(model, []).append((n, 100.0 * r["mfu"]))
    return line_svg(series, "scaling model: MFU of the best layout", "GPUs", "MFU (%)")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("result")
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    res = json.load(open(args.result))
    if isinstance(res, list):
        svg = scaling_chart(res)
    else:
        svg = ladder_chart(res) if "rows" in res else profile_chart(res)
    with open(args.out, "w") as f:
        f.write(svg)


if __name__ == "__main__":
    main()
