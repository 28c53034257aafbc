"""Allreduce sweep: every variant vs NCCL, 1 KB - 1 GB, schema-A CSV.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m results_b200.bench.allreduce_sweep \
        --variants nccl,oneshot,twoshot,nvls,ring,rhd,compressed --csv out.csv

The B200 counterpart of single_node_nccl_allreduce_benchmark/benchmark_both.py
of the reference (modes :372-383, CSV :644-687): the same CSV columns and
variant labels (Naive, N2Shot, Ring, RHD, 2Shot, P2P, RingP2P, Comp, NoSize,
plus OneShot, NVLS, NVLSOneShot, CompNative). Differences, on purpose:
device time is measured with CUDA events on every rank and the max over
ranks is reported (the reference timed rank 0 only); the per-iteration
random refill is excluded unless --include-fill is given; the compressed
ratio column is the measured ratio.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import time

import torch
import torch.distributed as dist

from ..utils import csvfmt

LABELS = {
    "nccl": "NCCL", "naive": "Naive", "naive_twoshot": "N2Shot", "ring_sendrecv": "Ring",
    "rhd_sendrecv": "RHD", "twoshot_collective": "2Shot", "twoshot": "P2P", "ring": "RingP2P",
    "compressed_ring": "Comp", "compressed_twoshot": "NoSize", "oneshot": "OneShot", "nvls": "NVLS",
    "nvls_oneshot": "NVLSOneShot", "rhd": "RHDP2P", "compressed": "CompNative",
    "compressed_hybrid": "CompHybrid",
    "multichannel_ring": "MCRing", "copy_engine": "P2PnoPA", "ll": "LL", "auto": "Auto", "ce": "MemcpyP2P",
}
NATIVE = {"oneshot", "twoshot", "nvls", "nvls_oneshot", "ring", "rhd", "ll", "auto", "ce"}
HOST = {"naive", "naive_twoshot", "ring_sendrecv", "rhd_sendrecv", "twoshot_collective", "multichannel_ring"}


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--variants", default="nccl,oneshot,twoshot,nvls,nvls_oneshot,ring,rhd,compressed")
    ap.add_argument("--min-bytes", type=int, default=1 << 10)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--include-fill", action="store_true")
    ap.add_argument("--check", action="store_true",
                    help="compare each variant's whole output with the fp32 rank-order sum rounded once; "
                         "the check column is the largest distance in ulps (0 = bit-exact), max over ranks")
    ap.add_argument("--graph", action="store_true",
                    help="capture the timed iterations of NCCL and the native kernels in one CUDA graph "
                         "(device time without per-call host overhead); host-staged variants stay eager")
    ap.add_argument("--csv", default=None)
    ap.add_argument("--json", default=None)
    return ap.parse_args()


def _max(v, ctrl):
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctrl)
    return float(t.item())


def _accuracy(y, n, dtype, world):
    """(largest ulp distance, largest |error| / max |sum|) of the whole output
    against the fp32 rank-order sum of every rank's input (regenerated from
    the seeds) rounded once. The ulp distance is given for 16-bit types only:
    for fp32 outputs near-cancelling sums make it meaningless."""
    acc = torch.zeros(n, device="cuda")
    for r in range(world):
        gg = torch.Generator(device="cuda").manual_seed(100 + r)
        acc += (torch.randn(n, device="cuda", generator=gg) * 1e-2).to(dtype).float()
    ref = acc.to(dtype)
    rel = float((y[:n].float() - acc).abs().max().item()) / max(float(acc.abs().max().item()), 1e-30)
    del acc
    if y.element_size() != 2:
        return None, rel
    u = y[:n].view(torch.int16).to(torch.int32)
    v = ref.view(torch.int16).to(torch.int32)
    u = torch.where(u < 0, -(u & 0x7FFF), u)
    v = torch.where(v < 0, -(v & 0x7FFF), v)
    return int((u - v).abs().max().item()), rel


def _capture(fn, fill, iters: int):
    """One CUDA graph of `iters` back-to-back calls (plus the input refill when timed)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for _ in range(iters):
            if fill:
                fill()
            fn()
    torch.cuda.current_stream().wait_stream(side)
    return g


def main():
    a = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=300))
    ctrl = dist.new_group(backend="gloo")
    import results_b200 as lz
    from results_b200.config import Config, MiB
    from results_b200.parallel import compressed as cz
    from results_b200.parallel import sendrecv, tuning

    dtype = getattr(torch, a.dtype)
    es = torch.empty((), dtype=dtype).element_size()
    variants = a.variants.split(",")
    stage = max(a.max_bytes + 64 * MiB, cz.stage_bytes_needed(a.max_bytes // es, dtype, world) + 64 * MiB) \
        if any(v.startswith("compressed") for v in variants) else a.max_bytes + 64 * MiB
    comm = lz.init(config=Config(user_bytes=2 * a.max_bytes + 64 * MiB, stage_bytes=stage,
                                 oneshot_bytes=8 * MiB))
    sizes = []
    s = a.min_bytes
    while s <= a.max_bytes:
        sizes.append(s)
        s *= 2
    rows = []
    for nbytes in sizes:
        n = nbytes // es
        comm.reset_alloc()
        xs = comm.empty(n, dtype)
        ys = comm.empty(n, dtype)
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        src = (torch.randn(n, device="cuda", generator=g) * 1e-2).to(dtype)
        res = {}
        for v in variants:
            if v in ("nvls", "nvls_oneshot") and not comm.has_multicast:
                continue
            if v in ("oneshot", "nvls_oneshot") and nbytes > 8 * MiB:
                continue
            if v == "ll" and (nbytes > 256 * 1024 or nbytes % 16):
                continue
            if v in ("rhd", "rhd_sendrecv") and world & (world - 1):
                continue
            xs.copy_(src)
            if v == "nccl":
                buf = src.clone()
                fn = lambda: dist.all_reduce(buf)
            elif v == "auto":
                algo = tuning.choose(nbytes, world, comm.has_multicast, symmetric=True, out_of_place=True)
                fn = lambda algo=algo: comm.allreduce_(xs, ys, algo=algo)
            elif v == "ce" and nbytes % (16 * world):
                continue
            elif v in NATIVE:
                fn = lambda v=v: comm.allreduce_(xs, ys, algo=v)
            elif v == "compressed":
                fn = lambda: cz.compressed_allreduce(xs, ys, comm=comm)
            elif v == "compressed_hybrid":
                fn = lambda: cz.compressed_allreduce(xs, ys, comm=comm, hybrid=True)
            elif v in HOST:
                buf = src.clone()
                fn = lambda v=v: sendrecv.allreduce(buf, v)
            elif v in ("compressed_twoshot", "compressed_ring"):
                buf = src.clone()
                fn = lambda v=v: cz.VARIANTS[v](buf)
            else:
                continue
            fill = (lambda: xs.copy_(src)) if a.include_fill else None
            for _ in range(a.warmup):
                if fill:
                    fill()
                fn()
            torch.cuda.synchronize()
            graph = None
            if a.graph and v not in HOST:
                graph = _capture(fn, fill, a.iters)
                graph.replay()  # warm the graph once (same collective count on every rank)
                torch.cuda.synchronize()
            dist.barrier(group=ctrl)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            t0 = time.perf_counter()
            if graph is not None:
                graph.replay()
            else:
                for _ in range(a.iters):
                    if fill:
                        fill()
                    fn()
            e1.record()
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            cuda_ms = _max(e0.elapsed_time(e1) / a.iters, ctrl)
            wall_ms = _max((t1 - t0) * 1e3 / a.iters, ctrl)
            comm.check()
            del graph  # graphs holding NCCL work are released before the group is destroyed
            ok = None
            if a.check and v in NATIVE | {"compressed", "compressed_hybrid", "nccl"}:
                xs.copy_(src)
                if v == "nccl":
                    buf.copy_(src)
                fn()
                torch.cuda.synchronize()
                ulp, rel = _accuracy(buf if v == "nccl" else ys, n, dtype, world)
                ok = (None if ulp is None else _max(float(ulp), ctrl), _max(rel, ctrl))
            ratio = None
            if v == "compressed" and rank == 0:
                ratio = lz.ops.codec.compression_ratio(src) if hasattr(lz, "ops") else None
            res[v] = (cuda_ms, wall_ms, ok, ratio)
        if rank == 0:
            base = res.get("nccl")
            for v, (cms, wms, ok, ratio) in res.items():
                for metric, ms, bms in (("wall_ms", wms, base[1] if base else None),
                                        ("cuda_ms", cms, base[0] if base else None)):
                    algbw = nbytes / (ms * 1e-3) / 1e9
                    busf = 2 * (world - 1) / world if world > 1 else 1.0
                    row = {
                        "metric": metric, "size_label": csvfmt.size_label(nbytes), "size_bytes": nbytes,
                        "world_size": world, "variant": LABELS.get(v, v), "nccl_ms": round(bms, 5) if bms else "",
                        "variant_ms": round(ms, 5),
                        "variant_vs_nccl_pct": round(100 * bms / ms, 1) if bms else "",
                        "nccl_algbw_GBps": round(nbytes / (bms * 1e-3) / 1e9, 3) if bms else "",
                        "variant_algbw_GBps": round(algbw, 3),
                        "nccl_busbw_GBps": round(nbytes / (bms * 1e-3) / 1e9 * busf, 3) if bms else "",
                        "variant_busbw_GBps": round(algbw * busf, 3),
                        "comp_ratio": round(ratio, 4) if ratio else "",
                        "max_ulp": "" if ok is None or ok[0] is None else int(ok[0]),
                        "max_rel_err": "" if ok is None else f"{ok[1]:.3g}",
                    }
                    rows.append(row)
            line = " ".join(f"{LABELS.get(v, v)}={nbytes / (r[0] * 1e-3) / 1e9 * (2 * (world - 1) / world if world > 1 else 1):.1f}"
                            for v, r in res.items())
            print(f"[{csvfmt.size_label(nbytes):>7}] busbw GB/s: {line}", flush=True)
        del xs, ys, src
    if rank == 0 and a.csv:
        wall = [r for r in rows if r["metric"] == "wall_ms"]
        cuda = [r for r in rows if r["metric"] == "cuda_ms"]
        header = csvfmt.SCHEMA_A + (["max_ulp", "max_rel_err"] if a.check else [])
        csvfmt.write_rows(a.csv, header, rows, blocks=[wall, cuda])
        csvfmt.write_sidecar(a.csv, {"bench": "allreduce_sweep", "world": world, "dtype": a.dtype,
                                     "iters": a.iters, "warmup": a.warmup, "include_fill": a.include_fill,
                                     "multicast": comm.has_multicast,
                                     "graph": a.graph, "check": "whole output vs the fp32 rank-order sum rounded once: max ulp (16-bit types) and "
                                              "max |error| / max |sum|"
                                     if a.check else None,
                                     "timing": "CUDA events per rank, max over ranks" +
                                               ("; timed iterations replayed from one CUDA graph" if a.graph else "")})
    if rank == 0 and a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f)
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
