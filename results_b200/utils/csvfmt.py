"""CSV schemas written by the benchmark drivers, column for column the same as
the reference's result files so its plotting and parsing scripts apply.

A  -- allreduce driver, single_node_nccl_allreduce_benchmark/benchmark_both.py:649-687
A' -- older allreduce tables (single_node_nccl_allreduce_benchmark/two-shot.csv:1)
B  -- p2p send bench (raw/result_bf16_split_rank0.csv:1)
B' -- weight-update bench (raw/GLM9B-0414_split_rank0.csv:1)
C  -- NCCL send/recv bench (back_up/nccl_send_recv_bench.py:67)
D  -- codec bench (raw/dietgpu_walltime_float16.csv:1)
"""
from __future__ import annotations

import csv
import json
import os
import subprocess
import time

SCHEMA_A = ["metric", "size_label", "size_bytes", "world_size", "variant", "nccl_ms", "variant_ms",
            "variant_vs_nccl_pct", "nccl_algbw_GBps", "variant_algbw_GBps", "nccl_busbw_GBps",
            "variant_busbw_GBps", "comp_ratio"]
SCHEMA_A2 = ["size_label", "size_bytes", "world_size", "variant", "cuda_ms", "wall_ms",
             "cuda_vs_nccl_pct", "wall_vs_nccl_pct", "cuda_algbw_GBps", "cuda_busbw_GBps",
             "wall_algbw_GBps", "wall_busbw_GBps", "comp_ratio"]
SCHEMA_B = ["role", "size_bytes", "size_pretty", "gbps", "gb_sec"]
SCHEMA_B2 = ["role", "mode", "size_bytes", "size_pretty", "gbps", "gb_sec", "iters", "rank", "world_size"]
SCHEMA_C = ["data_size_MB", "latency_sec", "throughput_GBps"]
SCHEMA_D = ["Data size", "size_bytes", "comp_time_ms", "decomp_time_ms", "comp_throughput_gb_s",
            "decomp_throughput_gb_s", "compressed_bytes", "compression_ratio"]


def size_label(nbytes: int) -> str:
    for unit, div in (("GB", 1 << 30), ("MB", 1 << 20), ("KB", 1 << 10)):
        if nbytes >= div and nbytes % div == 0:
            return f"{nbytes // div} {unit}"
    return f"{nbytes} B"


def write_rows(path: str, header: list[str], rows: list[dict], blocks: list[list[dict]] | None = None) -> None:
    """Write `rows` (or several blank-line separated blocks) under `header`."""
    os.makedirs(os.path.dirname(os.path.abspath(path)) or ".", exist_ok=True)
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=header, extrasaction="ignore")
        w.writeheader()
        if blocks is None:
            blocks = [rows]
        for i, blk in enumerate(blocks):
            if i:
                f.write("\n")
            for r in blk:
                w.writerow(r)


def git_sha() -> str | None:
    """HEAD of the source tree; LZ_GIT_SHA overrides it (a copy of the tree
    without its .git directory, e.g. on a remote benchmark machine)."""
    env = os.environ.get("LZ_GIT_SHA")
    if env:
        return env
    try:
        return subprocess.check_output(["git", "rev-parse", "HEAD"], stderr=subprocess.DEVNULL,
                                       cwd=os.path.dirname(os.path.abspath(__file__))).decode().strip()
    except Exception:
        return None


def write_sidecar(csv_path: str, meta: dict) -> str:
    """JSON sidecar next to a CSV: environment, git SHA, clocks, timing method."""
    import torch

    meta = dict(meta)
    meta.setdefault("time", time.time())
    meta.setdefault("git_sha", git_sha())
    meta.setdefault("torch", torch.__version__)
    if torch.cuda.is_available():
        meta.setdefault("gpu", torch.cuda.get_device_name())
    side = os.path.splitext(csv_path)[0] + ".json"
    with open(side, "w") as f:
        json.dump(meta, f, indent=1, default=str)
    return side
