"""All-to-all bench: NCCL all_to_all_single vs the native raw and compressed
kernels, per total message size (bytes each rank sends, all chunks).

    torchrun --nproc-per-node 8 -m results_b200.bench.alltoall_bench --csv a2a.csv

Reference counterpart: the LZip-NCCL vs NCCL all-to-all comparison of
plot/cccl_alltoall.py:7-16 (1 GB: 5.278 vs 4.482 GB/s on its link). Times are
CUDA events per rank, max over ranks; algbw = bytes sent per rank / time,
busbw = algbw x (W-1)/W. Data: bf16 N(0, 0.02) from a fixed seed per rank.
"""
from __future__ import annotations

import argparse
import datetime
import os

import torch
import torch.distributed as dist

from ..utils import csvfmt

HEADER = ["size_bytes", "size_label", "world_size", "variant", "ms", "algbw_GBps", "busbw_GBps", "check"]


def _max(v: float, group) -> float:
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--variants", default="nccl,raw,raw_symmetric,compressed")
    ap.add_argument("--min-bytes", type=int, default=1 << 20)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--csv", default=None)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()),
                            timeout=datetime.timedelta(seconds=300))
    ctrl = dist.new_group(backend="gloo")
    import results_b200 as lz
    from results_b200.config import Config, MiB
    from results_b200.parallel import alltoall

    dtype = torch.bfloat16
    stage = alltoall.stage_bytes_needed(a.max_bytes // 2, dtype, world, True) + 64 * MiB
    comm = lz.init(config=Config(user_bytes=a.max_bytes + 64 * MiB, stage_bytes=max(stage, a.max_bytes + 64 * MiB)))
    rows = []
    size = a.min_bytes
    while size <= a.max_bytes:
        n = size // 2 // world * world
        g = torch.Generator(device="cuda").manual_seed(500 + rank)
        x = (torch.randn(n, device="cuda", generator=g) * 0.02).to(dtype)
        comm.reset_alloc()
        sym = comm.empty(n, dtype)
        plain = torch.empty_like(x)
        ref = torch.empty_like(x)
        dist.all_to_all_single(ref, x)
        for v in a.variants.split(","):
            if v == "nccl":
                fn = lambda: dist.all_to_all_single(plain, x)  # noqa: E731
                res = plain
            elif v == "raw":
                fn = lambda: alltoall.all_to_all(x, plain, comm=comm)  # noqa: E731
                res = plain
            elif v == "raw_symmetric":
                fn = lambda: alltoall.all_to_all(x, sym, comm=comm)  # noqa: E731
                res = sym
            elif v == "compressed":
                fn = lambda: alltoall.all_to_all(x, plain, compress=True, comm=comm)  # noqa: E731
                res = plain
            else:
                continue
            for _ in range(a.warmup):
                fn()
            torch.cuda.synchronize()
            dist.barrier(group=ctrl)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            comm.check()
            ms = _max(e0.elapsed_time(e1) / a.iters, ctrl)
            ok = bool(torch.equal(res, ref))
            nbytes = n * 2
            algbw = nbytes / (ms * 1e-3) / 1e9
            rows.append({"size_bytes": nbytes, "size_label": csvfmt.size_label(nbytes), "world_size": world,
                         "variant": v, "ms": round(ms, 5), "algbw_GBps": round(algbw, 2),
                         "busbw_GBps": round(algbw * (world - 1) / world, 2), "check": ok})
            if rank == 0:
                print(f"[{csvfmt.size_label(nbytes):>7}] {v:14s} {ms * 1e3:10.1f} us  algbw {algbw:8.1f} GB/s  "
                      f"exact={ok}", flush=True)
        del x, plain, ref
        size *= 2
    if rank == 0 and a.csv:
        csvfmt.write_rows(a.csv, HEADER, rows)
        csvfmt.write_sidecar(a.csv, {"bench": "alltoall", "world": world, "dtype": "bfloat16",
                                     "timing": "CUDA events per rank, max over ranks"})
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
