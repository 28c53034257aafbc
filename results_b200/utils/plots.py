"""Dependency-free SVG charts of the benchmark CSVs.

The reference renders its figures with matplotlib/seaborn
(plot/plot_common.py:1-122 and plot/*.py -> fig/*.pdf). matplotlib is not
available in this image, so the same figures (bandwidth vs size per
variant, grouped bars per configuration) are written as standalone SVG.

    python -m results_b200.utils.plots sweep out.csv fig.svg   # schema-A allreduce sweep (bus GB/s)
    python -m results_b200.utils.plots latency out.csv fig.svg # the same, time per call (log)
    python -m results_b200.utils.plots kv kv.csv fig.svg       # KV-cache transfer latency vs tokens
    python -m results_b200.utils.plots weights fig.svg a.json b.json  # weight-update bars
    python -m results_b200.utils.plots xy in.csv fig.svg X Y SERIES [TITLE]  # any CSV
    python -m results_b200.utils.plots codec codec.csv fig.svg # schema-D codec table
"""
from __future__ import annotations

import csv
import math
import sys

PALETTE = ["#1f77b4", "#d62728", "#2ca02c", "#ff7f0e", "#9467bd", "#8c564b", "#e377c2", "#7f7f7f",
           "#bcbd22", "#17becf"]


def _esc(s) -> str:
    return str(s).replace("&", "&amp;").replace("<", "&lt;").replace(">", "&gt;")


def line_chart(series: dict, path: str, title: str = "", xlabel: str = "", ylabel: str = "",
               logx: bool = True, width: int = 760, height: int = 440, logy: bool = False) -> str:
    """series: {label: [(x, y), ...]} -> SVG file (log2 x axis; optional log10 y axis)."""
    pts = [p for s in series.values() for p in s if p[1] is not None]
    if not pts:
        raise ValueError("no data")
    fx = (lambda v: math.log2(v)) if logx else (lambda v: v)
    xs = [fx(p[0]) for p in pts]
    x0, x1 = min(xs), max(xs)
    y1 = max(p[1] for p in pts) * 1.08 or 1.0
    L, R, T, B = 70, 170, 40, 60
    W, H = width - L - R, height - T - B
    X = lambda v: L + (fx(v) - x0) / ((x1 - x0) or 1) * W
    if logy:
        ly0 = math.floor(math.log10(max(min(p[1] for p in pts), 1e-12)))
        ly1 = math.ceil(math.log10(y1))
        Y = lambda v: T + H - (math.log10(max(v, 1e-12)) - ly0) / ((ly1 - ly0) or 1) * H
    else:
        Y = lambda v: T + H - v / y1 * H
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" font-family="sans-serif" font-size="12">',
           f'<rect width="{width}" height="{height}" fill="white"/>',
           f'<text x="{width / 2}" y="22" text-anchor="middle" font-size="15">{_esc(title)}</text>',
           f'<line x1="{L}" y1="{T + H}" x2="{L + W}" y2="{T + H}" stroke="black"/>',
           f'<line x1="{L}" y1="{T}" x2="{L}" y2="{T + H}" stroke="black"/>']
    ticks = [10.0 ** e for e in range(ly0, ly1 + 1)] if logy else [y1 * k / 5 for k in range(6)]
    for v in ticks:
        out.append(f'<line x1="{L}" y1="{Y(v):.1f}" x2="{L + W}" y2="{Y(v):.1f}" stroke="#ddd"/>')
        out.append(f'<text x="{L - 6}" y="{Y(v) + 4:.1f}" text-anchor="end">{v:g}</text>')
    xticks = sorted({p[0] for p in pts})
    step = max(1, len(xticks) // 8)
    for xv in xticks[::step]:
        lab = xv
        if logx:
            for unit, div in (("G", 1 << 30), ("M", 1 << 20), ("K", 1 << 10)):
                if xv >= div:
                    lab = f"{xv / div:g}{unit}"
                    break
        out.append(f'<text x="{X(xv):.1f}" y="{T + H + 18}" text-anchor="middle">{_esc(lab)}</text>')
    out.append(f'<text x="{L + W / 2}" y="{height - 15}" text-anchor="middle">{_esc(xlabel)}</text>')
    out.append(f'<text x="18" y="{T + H / 2}" text-anchor="middle" transform="rotate(-90 18 {T + H / 2})">{_esc(ylabel)}</text>')
    for i, (lab, s) in enumerate(series.items()):
        s = sorted((p for p in s if p[1] is not None), key=lambda p: p[0])
        col = PALETTE[i % len(PALETTE)]
        d = " ".join(f"{'M' if j == 0 else 'L'}{X(x):.1f},{Y(y):.1f}" for j, (x, y) in enumerate(s))
        out.append(f'<path d="{d}" fill="none" stroke="{col}" stroke-width="2"/>')
        for x, y in s:
            out.append(f'<circle cx="{X(x):.1f}" cy="{Y(y):.1f}" r="2.5" fill="{col}"/>')
        ly = T + 14 + 18 * i
        out.append(f'<rect x="{L + W + 15}" y="{ly - 9}" width="12" height="12" fill="{col}"/>')
        out.append(f'<text x="{L + W + 32}" y="{ly + 1}">{_esc(lab)}</text>')
    out.append("</svg>")
    with open(path, "w") as f:
        f.write("\n".join(out))
    return path


def sweep_chart(csv_path: str, svg_path: str, metric: str = "cuda_ms", bus: bool = True) -> str:
    series: dict = {}
    with open(csv_path) as f:
        for r in csv.DictReader(f):
            if not r.get("metric") or r["metric"] != metric:
                continue
            key = "variant_busbw_GBps" if bus else "variant_algbw_GBps"
            series.setdefault(r["variant"], []).append((int(r["size_bytes"]), float(r[key])))
            if r.get("nccl_busbw_GBps"):
                series.setdefault("NCCL", [])
    ws = ""
    with open(csv_path) as f:
        for r in csv.DictReader(f):
            if r.get("world_size"):
                ws = r["world_size"]
                break
    return line_chart(series, svg_path, title=f"allreduce {'bus' if bus else 'alg'} bandwidth, {ws} x B200",
                      xlabel="message size", ylabel="GB/s")


def sweep_latency_chart(csv_path: str, svg_path: str, metric: str = "cuda_ms") -> str:
    """Per-call time (us, log scale) vs message size for every variant."""
    series: dict = {}
    ws = ""
    with open(csv_path) as f:
        for r in csv.DictReader(f):
            if r.get("metric") != metric:
                continue
            ws = r.get("world_size", ws)
            series.setdefault(r["variant"], []).append((int(r["size_bytes"]), float(r["variant_ms"]) * 1e3))
    return line_chart(series, svg_path, title=f"allreduce time per call, {ws} x B200",
                      xlabel="message size", ylabel="us (log)", logy=True)


def bar_chart(groups: dict, path: str, title: str = "", ylabel: str = "", width: int = 760,
              height: int = 440) -> str:
    """groups: {group label: {series label: value}} -> grouped-bar SVG."""
    labels = []
    for g in groups.values():
        for k in g:
            if k not in labels:
                labels.append(k)
    vmax = max((v for g in groups.values() for v in g.values() if v is not None), default=1.0) * 1.1 or 1.0
    L, R, T, B = 70, 170, 40, 70
    W, H = width - L - R, height - T - B
    gw = W / max(1, len(groups))
    bw = gw * 0.8 / max(1, len(labels))
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" font-family="sans-serif" font-size="12">',
           f'<rect width="{width}" height="{height}" fill="white"/>',
           f'<text x="{width / 2}" y="22" text-anchor="middle" font-size="15">{_esc(title)}</text>',
           f'<line x1="{L}" y1="{T + H}" x2="{L + W}" y2="{T + H}" stroke="black"/>',
           f'<line x1="{L}" y1="{T}" x2="{L}" y2="{T + H}" stroke="black"/>']
    for k in range(6):
        v = vmax * k / 5
        y = T + H - v / vmax * H
        out.append(f'<line x1="{L}" y1="{y:.1f}" x2="{L + W}" y2="{y:.1f}" stroke="#ddd"/>')
        out.append(f'<text x="{L - 6}" y="{y + 4:.1f}" text-anchor="end">{v:.3g}</text>')
    for gi, (gl, g) in enumerate(groups.items()):
        x0 = L + gi * gw + gw * 0.1
        for si, sl in enumerate(labels):
            v = g.get(sl)
            if v is None:
                continue
            h = v / vmax * H
            out.append(f'<rect x="{x0 + si * bw:.1f}" y="{T + H - h:.1f}" width="{bw * 0.9:.1f}" height="{h:.1f}" '
                       f'fill="{PALETTE[si % len(PALETTE)]}"/>')
        out.append(f'<text x="{L + gi * gw + gw / 2:.1f}" y="{T + H + 18}" text-anchor="middle">{_esc(gl)}</text>')
    out.append(f'<text x="18" y="{T + H / 2}" text-anchor="middle" transform="rotate(-90 18 {T + H / 2})">{_esc(ylabel)}</text>')
    for si, sl in enumerate(labels):
        ly = T + 14 + 18 * si
        out.append(f'<rect x="{L + W + 15}" y="{ly - 9}" width="12" height="12" fill="{PALETTE[si % len(PALETTE)]}"/>')
        out.append(f'<text x="{L + W + 32}" y="{ly + 1}">{_esc(sl)}</text>')
    out.append("</svg>")
    with open(path, "w") as f:
        f.write("\n".join(out))
    return path


def weight_update_chart(json_paths: list, svg_path: str) -> str:
    """Seconds per update by mode, one group per weight_update JSON (model x world)."""
    import json as _json

    groups = {}
    for jp in json_paths:
        with open(jp) as f:
            d = _json.load(f)
        groups[f"{d.get('model')} x{d.get('world')}"] = {m: r["sec"] for m, r in d["results"].items()}
    return bar_chart(groups, svg_path, title="RL weight update, seconds per update (lower is better)",
                     ylabel="s")


def kv_chart(csv_path: str, svg_path: str) -> str:
    """KV-cache transfer latency (ms) vs input tokens for every mode column."""
    series: dict = {}
    with open(csv_path) as f:
        for r in csv.DictReader(f):
            tok = int(r["Input Token"])
            for k, v in r.items():
                if k.endswith("(ms)") and v not in ("", None):
                    series.setdefault(k.replace(" latency (ms)", "").replace(" kv cache transfer", ""), []).append(
                        (tok, float(v)))
    return line_chart(series, svg_path, title="prefill -> decode KV-cache transfer, 2 x B200",
                      xlabel="input tokens", ylabel="ms")


def xy_chart(csv_path: str, svg_path: str, x: str, y: str, series: str, title: str = "",
             ylabel: str = "") -> str:
    """Generic line chart of one CSV: column `y` vs column `x`, one line per value of `series`."""
    data: dict = {}
    with open(csv_path) as f:
        for r in csv.DictReader(f):
            if r.get(x) in (None, "") or r.get(y) in (None, ""):
                continue
            data.setdefault(r[series], []).append((float(r[x]), float(r[y])))
    return line_chart(data, svg_path, title=title, xlabel=x, ylabel=ylabel or y)


def codec_chart(csv_path: str, svg_path: str) -> str:
    comp, dec = [], []
    with open(csv_path) as f:
        for r in csv.DictReader(f):
            comp.append((int(r["size_bytes"]), float(r["comp_throughput_gb_s"])))
            dec.append((int(r["size_bytes"]), float(r["decomp_throughput_gb_s"])))
    return line_chart({"compress": comp, "decompress": dec}, svg_path, title="LZC1 codec throughput",
                      xlabel="input size", ylabel="GB/s")


if __name__ == "__main__":
    kind, src, dst = sys.argv[1:4]
    if kind == "xy":  # plots xy in.csv out.svg X Y SERIES [TITLE]
        xy_chart(src, dst, sys.argv[4], sys.argv[5], sys.argv[6], title=sys.argv[7] if len(sys.argv) > 7 else "")
        print(dst)
        sys.exit(0)
    if kind == "weights":  # plots weights out.svg a.json b.json ...
        weight_update_chart(sys.argv[3:], src)
        print(src)
        sys.exit(0)
    {"sweep": sweep_chart, "latency": sweep_latency_chart, "codec": codec_chart, "kv": kv_chart}[kind](src, dst)
    print(dst)
