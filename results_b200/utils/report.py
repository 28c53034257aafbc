"""Markdown summary tables from the measured CSV / JSON files.

    python -m results_b200.utils.report results/

Reads the files the benchmark drivers write (schema-A allreduce sweeps,
weight-update JSON, KV-transfer and all-to-all CSVs) and prints the tables
the documentation quotes, so every quoted number can be regenerated from the
data it came from.
"""
from __future__ import annotations

import csv
import glob
import json
import os
import re
import sys

SIZES = ["1 KB", "64 KB", "256 KB", "1 MB", "4 MB", "16 MB", "64 MB", "256 MB", "1 GB"]


def sweep_times(path: str) -> dict:
    """{size label: {variant: us}} from the cuda_ms rows of a schema-A CSV."""
    out: dict = {}
    with open(path) as f:
        for r in csv.DictReader(f):
            if r.get("metric") != "cuda_ms":
                continue
            out.setdefault(r["size_label"], {})[r["variant"]] = float(r["variant_ms"]) * 1e3
    return out


def allreduce_table(paths: dict) -> str:
    """paths: {world: csv}. Auto vs NCCL per size, with the speed-up."""
    data = {w: sweep_times(p) for w, p in sorted(paths.items())}
    head = "| size | " + " | ".join(f"{w} GPUs auto / NCCL (us)" for w in data) + " |"
    lines = [head, "|---|" + "---|" * len(data)]
    for s in SIZES:
        cells = []
        for w, d in data.items():
            r = d.get(s, {})
            if "Auto" in r and "NCCL" in r:
                cells.append(f"{r['Auto']:.1f} / {r['NCCL']:.1f} ({r['NCCL'] / r['Auto']:.2f}x)")
            else:
                cells.append("")
        lines.append(f"| {s} | " + " | ".join(cells) + " |")
    worst = min(((d[s]["NCCL"] / d[s]["Auto"], w, s) for w, d in data.items() for s in d
                 if "Auto" in d[s] and "NCCL" in d[s]), default=None)
    if worst:
        lines.append(f"\nSmallest margin over NCCL: {worst[0]:.2f}x ({worst[1]} GPUs, {worst[2]}).")
    return "\n".join(lines)


LINK_GBPS = 770.0  # measured peer-copy bandwidth per direction on this pool's B200s


def roofline_table(paths: dict, size: str = "1 GB") -> str:
    """Two-shot and NVLS at `size`: NVLink bytes per GPU per direction over the
    measured link bandwidth, against the measured time. Two-shot moves
    2(N-1)/N n each way; NVLS (1 + 1/N) n (switch-side reduce, multicast store)."""
    lines = ["| algorithm | GPUs | bound (us) | measured (us) | of bound |", "|---|---|---|---|---|"]
    n = 1 << 30 if size == "1 GB" else None
    for w, p in sorted(paths.items()):
        d = sweep_times(p).get(size, {})
        for label, factor in (("P2P", 2 * (w - 1) / w), ("NVLS", 1 + 1 / w)):
            if label in d and n:
                bound = factor * n / (LINK_GBPS * 1e9) * 1e6
                lines.append(f"| {'two-shot' if label == 'P2P' else 'NVLS'} | {w} | {bound:.0f} | {d[label]:.0f} | "
                             f"{100 * bound / d[label]:.0f} % |")
    return "\n".join(lines)


def weight_table(paths: list) -> str:
    lines = ["| file | model | ranks | mode | s / update | GB/s per receiver | bit-exact |",
             "|---|---|---|---|---|---|---|"]
    for p in paths:
        with open(p) as f:
            d = json.load(f)
        for m, r in d.get("results", {}).items():
            lines.append(f"| {os.path.basename(p)} | {d.get('model')} | {d.get('world')} | {m} | {r['sec']:.4f} | "
                         f"{r['GBps_per_receiver']:.1f} | {r['bitexact']} |")
    return "\n".join(lines)


def csv_table(path: str, cols: list | None = None) -> str:
    with open(path) as f:
        rows = list(csv.DictReader(f))
    if not rows:
        return ""
    cols = cols or list(rows[0].keys())
    lines = ["| " + " | ".join(cols) + " |", "|" + "---|" * len(cols)]
    for r in rows:
        lines.append("| " + " | ".join(str(r.get(c, "")) for c in cols) + " |")
    return "\n".join(lines)


def main(argv=None) -> str:
    root = (argv or sys.argv[1:] or ["results"])[0]
    parts = []
    sweeps = {}
    for p in glob.glob(os.path.join(root, "csv", "allreduce_sweep_*xB200_graph.csv")):
        m = re.search(r"_(\d+)xB200", p)
        if m:
            sweeps[int(m.group(1))] = p
    if sweeps:
        parts.append("## Allreduce (CUDA-graph device time)\n\n" + allreduce_table(sweeps))
        parts.append("## Roofline, 1 GB (NVLink bytes per direction / 770 GB/s)\n\n" + roofline_table(sweeps))
    wj = sorted(glob.glob(os.path.join(root, "json", "weight_update_*.json")))
    if wj:
        parts.append("## Weight update\n\n" + weight_table(wj))
    for name, title in (("kv_transfer_2xB200.csv", "KV-cache transfer"), ("alltoall_8xB200.csv", "All-to-all")):
        p = os.path.join(root, "csv", name)
        if os.path.exists(p):
            parts.append(f"## {title}\n\n" + csv_table(p))
    text = "\n\n".join(parts)
    print(text)
    return text


if __name__ == "__main__":
    main()
