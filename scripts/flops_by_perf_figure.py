#!/usr/bin/env python
"""
Draw "training FLOPs versus benchmark score" as an SVG scatter plot with a logarithmic x axis (the role of the
reference's ``scripts/flops_by_perf_figure.py``, which hard-codes one paper figure; this one reads its points).

    python scripts/flops_by_perf_figure.py points.csv figure.svg [--title "..."] [--ylabel "Average accuracy"]
    python scripts/flops_by_perf_figure.py --flops-of OLMo2-7B-stage1 --tokens 4e12      # print 6·N·D-style training FLOPs

``points.csv`` has a header and the columns ``model,flops,score`` plus an optional ``group`` (one colour and legend
entry per group).  A ``flops`` cell may be a number or ``recipe:tokens`` (e.g. ``OLMo2-7B-stage1:4e12``), which is
expanded with the model's own FLOPs-per-token count (forward + backward, attention included).
"""
import argparse
import csv
import math
import sys
from pathlib import Path
from typing import Dict, List, Optional, Tuple

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

PALETTE = ["#0a3235", "#f0529c", "#105257", "#b11be8", "#ff9100", "#0fcb8c", "#265ed4", "#88000f"]


def training_flops(recipe: str, tokens: float) -> float:
    """FLOPs of training ``recipe``'s architecture on ``tokens`` tokens."""
    from olmo_b200.models.olmo import OLMo
    from olmo_b200.recipes import recipe_config

    cfg = recipe_config(recipe).model
    cfg.init_device = "meta"
    model = OLMo(cfg, init_params=False)
    return float(model.num_fwd_flops + model.num_bck_flops) * tokens


def read_points(path: Path) -> List[Dict[str, object]]:
    points = []
    with open(path, newline="") as f:
        for row in csv.DictReader(f):
            flops = row["flops"].strip()
            if ":" in flops:
                recipe, tokens = flops.rsplit(":", 1)
                value = training_flops(recipe, float(tokens))
            else:
                value = float(flops)
            points.append({"model": row["model"].strip(), "flops": value, "score": float(row["score"]), "group": (row.get("group") or "").strip()})
    if not points:
        raise ValueError(f"{path} has no rows")
    return points


def render_svg(points: List[Dict[str, object]], title: str = "", xlabel: str = "Approximate training FLOPs", ylabel: str = "Score",
               width: int = 860, height: int = 520, font_path: Optional[str] = None) -> str:
    left, right, top, bottom = 70, 200, 40, 60
    xs = [math.log10(p["flops"]) for p in points]  # type: ignore[arg-type]
    ys = [float(p["score"]) for p in points]  # type: ignore[arg-type]
    x0, x1 = math.floor(min(xs) * 2) / 2, math.ceil(max(xs) * 2) / 2
    if x0 == x1:
        x1 = x0 + 0.5
    pad = (max(ys) - min(ys)) * 0.08 or 1.0
    y0, y1 = min(ys) - pad, max(ys) + pad

    def px(x: float) -> float:
        return left + (x - x0) / (x1 - x0) * (width - left - right)

    def py(y: float) -> float:
        return height - bottom - (y - y0) / (y1 - y0) * (height - top - bottom)

    groups: List[str] = []
    for p in points:
        if p["group"] not in groups:
            groups.append(p["group"])  # type: ignore[arg-type]
    family = "sans-serif"
    font_face = ""
    if font_path:  # embed the font file so that the figure renders the same everywhere
        import base64

        data = base64.b64encode(Path(font_path).read_bytes()).decode()
        kind = "opentype" if str(font_path).lower().endswith(".otf") else "truetype"
        family = "FigureFont, sans-serif"
        font_face = f'<style>@font-face {{ font-family: FigureFont; src: url(data:font/{kind};base64,{data}) format("{kind}"); }}</style>'
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" font-family="{family}" font-size="12">',
           font_face, f'<rect width="{width}" height="{height}" fill="white"/>']
    if title:
        out.append(f'<text x="{width / 2}" y="22" text-anchor="middle" font-size="15">{title}</text>')
    tick = x0
    while tick <= x1 + 1e-9:  # one grid line per half decade
        x = px(tick)
        out.append(f'<line x1="{x:.1f}" y1="{top}" x2="{x:.1f}" y2="{height - bottom}" stroke="#ddd"/>')
        label = f"10^{tick:g}" if tick == int(tick) else ""
        out.append(f'<text x="{x:.1f}" y="{height - bottom + 18}" text-anchor="middle">{label}</text>')
        tick += 0.5
    for i in range(6):
        yv = y0 + (y1 - y0) * i / 5
        out.append(f'<line x1="{left}" y1="{py(yv):.1f}" x2="{width - right}" y2="{py(yv):.1f}" stroke="#ddd"/>')
        out.append(f'<text x="{left - 8}" y="{py(yv) + 4:.1f}" text-anchor="end">{yv:.1f}</text>')
    out.append(f'<rect x="{left}" y="{top}" width="{width - left - right}" height="{height - top - bottom}" fill="none" stroke="#333"/>')
    out.append(f'<text x="{(left + width - right) / 2}" y="{height - 14}" text-anchor="middle">{xlabel}</text>')
    out.append(f'<text x="18" y="{(top + height - bottom) / 2}" text-anchor="middle" transform="rotate(-90 18 {(top + height - bottom) / 2})">{ylabel}</text>')
    for p, x, y in zip(points, xs, ys):
        colour = PALETTE[groups.index(p["group"]) % len(PALETTE)]  # type: ignore[arg-type]
        out.append(f'<circle cx="{px(x):.1f}" cy="{py(y):.1f}" r="5" fill="{colour}"><title>{p["model"]}</title></circle>')
        out.append(f'<text x="{px(x) + 7:.1f}" y="{py(y) - 6:.1f}" font-size="10">{p["model"]}</text>')
    for i, group in enumerate(g for g in groups if g):
        y = top + 14 + 18 * i
        out.append(f'<circle cx="{width - right + 20}" cy="{y - 4}" r="5" fill="{PALETTE[groups.index(group) % len(PALETTE)]}"/>')
        out.append(f'<text x="{width - right + 32}" y="{y}">{group}</text>')
    out.append("</svg>")
    return "\n".join(out) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("points", nargs="?")
    ap.add_argument("output", nargs="?")
    ap.add_argument("--title", default="")
    ap.add_argument("--ylabel", default="Score")
    ap.add_argument("--flops-of", default=None, metavar="RECIPE")
    ap.add_argument("--tokens", type=float, default=None)
    ap.add_argument("--manrope-medium-font-path", "--font-path", dest="font_path", default=None,
                    help="a .ttf/.otf file to embed in the figure and use for all text (the published figure uses Manrope Medium)")
    args = ap.parse_args(argv)
    if args.flops_of:
        if args.tokens is None:
            ap.error("--flops-of needs --tokens")
        print(f"{training_flops(args.flops_of, args.tokens):.4e}")
        return 0
    if not args.points or not args.output:
        ap.error("points.csv and figure.svg are required")
    Path(args.output).write_text(render_svg(read_points(Path(args.points)), title=args.title, ylabel=args.ylabel, font_path=args.font_path))
    print(args.output)
    return 0


if __name__ == "__main__":
    sys.exit(main())
