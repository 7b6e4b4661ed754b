"""SVG charts of ladder / profile results (reference: make_charts.py, which needs matplotlib;
this writes plain SVG so it runs anywhere). The architecture label comes from the result
file's env info, never a hard-coded name.

    python -m llmt.bench.charts results/ladder_small.json --out results/ladder_small.svg
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


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("result")
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    res = json.load(open(args.result))
    svg = ladder_chart(res) if "rows" in res else profile_chart(res)
    with open(args.out, "w") as f:
        f.write(svg)


if __name__ == "__main__":
    main()
