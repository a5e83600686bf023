"""Bandwidth-versus-M figures from the sweep CSV, with B200 reference lines.

    python -m decode_opt_b200.plot [CSV ...] [--results DIR] [--out DIR]
        [--models id,...] [--steps 0-7] [--peaks MEASURED_PEAKS.json]
        [--tflops 4500] [--spec-gbps 8000]

The B200 counterpart of the reference's analysis/plot.py (its curve rule
:376-383 and reference lines :686-712, :206-232): one panel per model, x = M
(1..128, log2 axis), y = equivalent bandwidth (N*K + M*K + 2*M*N) / p50 in
GB/s, one curve per ladder step -- step 0 from the B2B protocol, later steps
from PDL (another protocol, marked with a dagger, only where that one is
missing) -- and three reference lines:

  * the B200 HBM3e spec, 8000 GB/s (solid);
  * the measured HBM peak, `hbm_gbs` of MEASURED_PEAKS.json (dashed; left
    out, with a note, when the file is absent -- never a made-up number);
  * the compute roof as an equivalent bandwidth,
    BW_cap(M) = min(spec, bytes(M) / t_floor(M)), t_floor = 2*M*N*K / FP8
    peak (dash-dot; B200 dense FP8, 4.5 PFLOP/s nominal by default).

The figures are SVG written directly (no plotting library in the image):
`fig_bw_vs_M_<model>.svg` per model and `fig_main_bw_vs_M.svg` with every
panel.
"""

from __future__ import annotations

import argparse
import csv
import glob
import json
import math
import os
import sys
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple
from xml.sax.saxutils import escape

SPEC_GBPS = 8000.0
FP8_DENSE_TFLOPS = 4500.0
M_MIN, M_MAX = 1, 128
STEP_COLORS = ("#9e9e9e", "#8d6e63", "#ffb300", "#7cb342", "#26a69a", "#42a5f5", "#d81b60", "#5e35b1")
COLOR_SPEC, COLOR_MEASURED, COLOR_ROOF = "#212121", "#c62828", "#6a1b9a"


def canon_protocol(step: int) -> str:
    """The protocol a step's curve is drawn from: B2B for step 0, PDL after."""
    return "B2B" if step == 0 else "PDL"


def moved_bytes(n: int, k: int, m: float) -> float:
    return float(n) * k + float(m) * k + 2.0 * m * n


def roof_gbps(m: float, n: int, k: int, tflops: float, spec: float) -> float:
    """min(spec, bytes(M) / t_floor(M)) with t_floor = 2*M*N*K / tflops."""
    t_floor = 2.0 * m * n * k / (tflops * 1e12)
    return min(spec, moved_bytes(n, k, m) / t_floor / 1e9)


@dataclass
class Curve:
    step: int
    name: str
    protocol: str
    fallback: bool
    points: List[Tuple[int, float]] = field(default_factory=list)   # (M, GB/s), M ascending


@dataclass
class ModelCurves:
    model: str
    n: int
    k: int
    curves: Dict[int, Curve] = field(default_factory=dict)


def _float(s: str) -> float:
    try:
        v = float(s)
    except (TypeError, ValueError):
        return float("nan")
    return v


def load_rows(paths: Sequence[str]) -> List[dict]:
    """Rows of the 16-column CSVs with a finite latency and pass != 0."""
    out = []
    for p in paths:
        with open(p, newline="") as f:
            for r in csv.DictReader(f):
                if r.get("pass", "na") == "0":
                    continue
                lat = _float(r.get("latency_us_p50"))
                if not (lat > 0 and math.isfinite(lat)):
                    continue
                out.append(r)
    return out


def build_curves(rows: Sequence[dict], steps: Optional[Sequence[int]] = None,
                 models: Optional[Sequence[str]] = None) -> List[ModelCurves]:
    """Per model and step, the best p50 per M under the step's protocol (or,
    where it has no row, the best other protocol, marked as a fallback);
    bandwidth recomputed from N, K, M and the p50."""
    by_key: Dict[Tuple[str, int, str, int], Tuple[float, dict]] = {}
    order: List[str] = []
    for r in rows:
        model, step, proto, m = r["model"], int(r["step"]), r["protocol"], int(r["M"])
        if steps is not None and step not in steps:
            continue
        if models and model not in models:
            continue
        if model not in order:
            order.append(model)
        lat = _float(r["latency_us_p50"])
        key = (model, step, proto, m)
        if key not in by_key or lat < by_key[key][0]:
            by_key[key] = (lat, r)
    out = []
    for model in (models or order):
        mc = None
        for step in sorted({k[1] for k in by_key if k[0] == model}):
            want = canon_protocol(step)
            ms = sorted({k[3] for k in by_key if k[0] == model and k[1] == step})
            pts, fallback, name, protos = [], False, "", set()
            for m in ms:
                hit = by_key.get((model, step, want, m))
                if hit is None:
                    alts = [v for k, v in by_key.items() if k[0] == model and k[1] == step and k[3] == m]
                    hit = min(alts, key=lambda v: v[0])
                    fallback = True
                lat, r = hit
                n, k = int(r["N"]), int(r["K"])
                if mc is None:
                    mc = ModelCurves(model, n, k)
                name = r.get("step_name", "")
                protos.add(r["protocol"])
                pts.append((m, moved_bytes(n, k, m) / (lat * 1e-6) / 1e9))
            if mc is not None and pts:
                mc.curves[step] = Curve(step, name, want if not fallback else "/".join(sorted(protos)), fallback, pts)
        if mc is not None:
            out.append(mc)
    return out


def measured_peak(path: Optional[str]) -> Tuple[Optional[float], str]:
    if not path:
        return None, "no measured peak given"
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), path
    except (OSError, ValueError, KeyError) as e:
        return None, f"measured peak unavailable ({type(e).__name__}: {path})"


# ---------------------------------------------------------------------------
# SVG
# ---------------------------------------------------------------------------

def _nice_step(span: float) -> float:
    raw = span / 6.0
    mag = 10 ** math.floor(math.log10(raw))
    for f in (1, 2, 2.5, 5, 10):
        if raw <= f * mag:
            return f * mag
    return 10 * mag


class Panel:
    def __init__(self, x0: float, y0: float, w: float, h: float, ymax: float):
        self.x0, self.y0, self.w, self.h, self.ymax = x0, y0, w, h, ymax

    def px(self, m: float) -> float:
        return self.x0 + (math.log2(m) - math.log2(M_MIN)) / (math.log2(M_MAX) - math.log2(M_MIN)) * self.w

    def py(self, v: float) -> float:
        return self.y0 + self.h - max(0.0, min(v, self.ymax)) / self.ymax * self.h


def _line(x1, y1, x2, y2, color, width=1.0, dash=None) -> str:
    d = f' stroke-dasharray="{dash}"' if dash else ""
    return (f'<line x1="{x1:.1f}" y1="{y1:.1f}" x2="{x2:.1f}" y2="{y2:.1f}" stroke="{color}" '
            f'stroke-width="{width}"{d}/>')


def _text(x, y, s, size=11, anchor="start", color="#212121", weight="normal") -> str:
    return (f'<text x="{x:.1f}" y="{y:.1f}" font-size="{size}" text-anchor="{anchor}" fill="{color}" '
            f'font-weight="{weight}" font-family="sans-serif">{escape(s)}</text>')


def panel_svg(p: Panel, mc: ModelCurves, spec: float, measured: Optional[float], tflops: float,
              title: str) -> List[str]:
    out = [f'<rect x="{p.x0:.1f}" y="{p.y0:.1f}" width="{p.w:.1f}" height="{p.h:.1f}" fill="white" '
           f'stroke="#424242" stroke-width="1"/>', _text(p.x0 + p.w / 2, p.y0 - 8, title, 13, "middle",
                                                         weight="bold")]
    step = _nice_step(p.ymax)
    v = 0.0
    while v <= p.ymax + 1e-9:
        y = p.py(v)
        out.append(_line(p.x0, y, p.x0 + p.w, y, "#eeeeee"))
        out.append(_text(p.x0 - 6, y + 4, f"{v:g}", 10, "end", "#616161"))
        v += step
    m = M_MIN
    while m <= M_MAX:
        x = p.px(m)
        out.append(_line(x, p.y0, x, p.y0 + p.h, "#eeeeee"))
        out.append(_text(x, p.y0 + p.h + 14, str(m), 10, "middle", "#616161"))
        m *= 2
    out.append(_text(p.x0 + p.w / 2, p.y0 + p.h + 30, "M (batch rows)", 11, "middle"))
    out.append(f'<text x="{p.x0 - 44:.1f}" y="{p.y0 + p.h / 2:.1f}" font-size="11" text-anchor="middle" '
               f'font-family="sans-serif" transform="rotate(-90 {p.x0 - 44:.1f} {p.y0 + p.h / 2:.1f})">'
               f'GB/s</text>')
    # reference lines
    ys = p.py(spec)
    out.append(f'<g class="ref-spec">{_line(p.x0, ys, p.x0 + p.w, ys, COLOR_SPEC, 1.6)}'
               f'{_text(p.x0 + p.w - 4, ys - 4, f"B200 HBM3e spec {spec:g} GB/s", 10, "end", COLOR_SPEC)}</g>')
    if measured:
        ym = p.py(measured)
        out.append(f'<g class="ref-measured">{_line(p.x0, ym, p.x0 + p.w, ym, COLOR_MEASURED, 1.6, "6,4")}'
                   f'{_text(p.x0 + p.w - 4, ym + 13, f"measured HBM peak {measured:.0f} GB/s", 10, "end", COLOR_MEASURED)}</g>')
    pts = []
    steps_m = 64
    for i in range(steps_m + 1):
        m = M_MIN * (M_MAX / M_MIN) ** (i / steps_m)
        cap = roof_gbps(m, mc.n, mc.k, tflops, spec)
        if cap < spec - 0.5:
            pts.append(f"{p.px(m):.1f},{p.py(cap):.1f}")
    if pts:
        out.append(f'<polyline class="ref-roof" points="{" ".join(pts)}" fill="none" stroke="{COLOR_ROOF}" '
                   f'stroke-width="1.6" stroke-dasharray="9,3,2,3"/>')
    # step curves
    for i, (step, c) in enumerate(sorted(mc.curves.items())):
        color = STEP_COLORS[step % len(STEP_COLORS)]
        poly = " ".join(f"{p.px(m):.1f},{p.py(v):.1f}" for m, v in c.points)
        out.append(f'<polyline class="step-{step}" points="{poly}" fill="none" stroke="{color}" '
                   f'stroke-width="2"/>')
        for m, v in c.points:
            out.append(f'<circle cx="{p.px(m):.1f}" cy="{p.py(v):.1f}" r="2.6" fill="{color}"/>')
    return out


def legend_svg(x: float, y: float, curves: Dict[int, Curve], measured: Optional[float], tflops: float,
               spec: float) -> List[str]:
    out = []
    for i, (step, c) in enumerate(sorted(curves.items())):
        color = STEP_COLORS[step % len(STEP_COLORS)]
        yy = y + 16 * i
        label = f"S{step} {c.name} ({c.protocol}{' †' if c.fallback else ''})"
        out.append(_line(x, yy, x + 22, yy, color, 2.5))
        out.append(_text(x + 28, yy + 4, label, 11))
    yy = y + 16 * len(curves) + 8
    out.append(_line(x, yy, x + 22, yy, COLOR_SPEC, 1.6))
    out.append(_text(x + 28, yy + 4, f"B200 HBM3e spec {spec:g} GB/s", 11))
    yy += 16
    if measured:
        out.append(_line(x, yy, x + 22, yy, COLOR_MEASURED, 1.6, "6,4"))
        out.append(_text(x + 28, yy + 4, f"measured HBM peak {measured:.0f} GB/s", 11))
        yy += 16
    out.append(_line(x, yy, x + 22, yy, COLOR_ROOF, 1.6, "9,3,2,3"))
    out.append(_text(x + 28, yy + 4, f"compute roof: min(spec, bytes/(2MNK / {tflops:g} TFLOP/s))", 11))
    return out


def figure(models: Sequence[ModelCurves], spec: float, measured: Optional[float], tflops: float,
           cols: int, title: str) -> str:
    pw, ph, mx, my = 420.0, 280.0, 80.0, 70.0
    rows_n = max(1, math.ceil((len(models) + 1) / cols))
    width = mx + cols * (pw + mx)
    height = 50 + rows_n * (ph + my + 20)
    vmax = max([spec, measured or 0.0] + [v for mc in models for c in mc.curves.values() for _, v in c.points])
    ymax = vmax * 1.08
    body = [_text(width / 2, 28, title, 16, "middle", weight="bold")]
    all_curves: Dict[int, Curve] = {}
    for i, mc in enumerate(models):
        r, c = divmod(i, cols)
        p = Panel(mx + c * (pw + mx), 60 + r * (ph + my + 20), pw, ph, ymax)
        body += panel_svg(p, mc, spec, measured, tflops, f"{mc.model} (N={mc.n}, K={mc.k})")
        for step, cv in mc.curves.items():
            all_curves.setdefault(step, cv)
    r, c = divmod(len(models), cols)
    body += legend_svg(mx + c * (pw + mx) + 10, 80 + r * (ph + my + 20), all_curves, measured, tflops, spec)
    return (f'<svg xmlns="http://www.w3.org/2000/svg" width="{width:.0f}" height="{height:.0f}" '
            f'viewBox="0 0 {width:.0f} {height:.0f}">\n<rect width="100%" height="100%" fill="white"/>\n'
            + "\n".join(body) + "\n</svg>\n")


def newest_csv(directory: str) -> Optional[str]:
    names = [p for p in glob.glob(os.path.join(directory, "bench_*.csv")) if not p.endswith("_detail.csv")]
    return max(names) if names else None


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("csv", nargs="*", help="16-column sweep CSVs (default: newest bench_*.csv in --results)")
    ap.add_argument("--results", default="results")
    ap.add_argument("--out", default=None, help="output directory (default: the first CSV's)")
    ap.add_argument("--models", default="", help="comma list (default: every model in the CSVs)")
    ap.add_argument("--steps", default="", help="e.g. 0-7 or 4,6,7 (default: all)")
    ap.add_argument("--peaks", default="MEASURED_PEAKS.json", help="JSON with hbm_gbs (measured line)")
    ap.add_argument("--tflops", type=float, default=FP8_DENSE_TFLOPS, help="FP8 peak for the compute roof")
    ap.add_argument("--spec-gbps", type=float, default=SPEC_GBPS)
    args = ap.parse_args(argv)
    paths = list(args.csv)
    if not paths:
        p = newest_csv(args.results)
        if p is None:
            print(f"[plot] no bench_*.csv in {args.results}", file=sys.stderr)
            return 2
        paths = [p]
    steps = None
    if args.steps:
        from .bench_decode import parse_int_ranges
        steps = parse_int_ranges(args.steps, 0, 7)
    models = [m for m in args.models.split(",") if m] or None
    curves = build_curves(load_rows(paths), steps, models)
    if not curves:
        print("[plot] no usable rows", file=sys.stderr)
        return 2
    measured, note = measured_peak(args.peaks)
    if measured is None:
        print(f"[plot] {note}: the measured line is left out", file=sys.stderr)
    out_dir = args.out or os.path.dirname(os.path.abspath(paths[0]))
    os.makedirs(out_dir, exist_ok=True)
    written = []
    for mc in curves:
        path = os.path.join(out_dir, f"fig_bw_vs_M_{mc.model}.svg")
        with open(path, "w") as f:
            f.write(figure([mc], args.spec_gbps, measured, args.tflops, 2,
                           f"{mc.model}: equivalent bandwidth vs M (B200)"))
        written.append(path)
    path = os.path.join(out_dir, "fig_main_bw_vs_M.svg")
    with open(path, "w") as f:
        f.write(figure(curves, args.spec_gbps, measured, args.tflops, 3,
                       "FP8 decode GEMM on B200: equivalent bandwidth vs M"))
    written.append(path)
    for p in written:
        print(p)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
