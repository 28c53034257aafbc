"""Codec throughput bench (schema D), the B200 counterpart of the reference's
dietgpu wall-time tables (csv/dietgpu_walltime_bfloat16_new.csv,
raw/dietgpu_walltime_float{16,32}.csv of the reference).

    python -m results_b200.bench.codec_bench --dtype bfloat16 --csv out.csv

Throughput = uncompressed bytes / device time (CUDA events, median of
--iters runs after --warmup). Inputs above 126 MB exceed L2; for smaller
inputs an L2-sized buffer is written between timed runs.
"""
from __future__ import annotations

import argparse
import statistics

import torch

from ..ops import codec
from ..utils import csvfmt

L2_FLUSH_BYTES = 256 << 20


def _time(fn, iters, warmup, flush):
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def make_data(n, dtype, dist="normal", std=0.02, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if dist == "normal":
        x = torch.randn(n, device="cuda", generator=g) * std
    elif dist == "activation":  # N(0,1) with 1% outliers x50 (activation-like)
        x = torch.randn(n, device="cuda", generator=g)
        m = torch.rand(n, device="cuda", generator=g) < 0.01
        x = torch.where(m, x * 50, x)
    else:
        raise ValueError(dist)
    if dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        return x.to(dtype)
    return x.to(dtype)


def run(sizes_mb, dtype, iters=10, warmup=3, dist="normal", std=0.02, nblocks=0, level="ans"):
    rows = []
    for mb in sizes_mb:
        nbytes = mb << 20
        es = torch.empty((), dtype=dtype).element_size()
        n = nbytes // es
        x = make_data(n, dtype, dist, std)
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda") if nbytes < (128 << 20) else None
        L = codec._native.cuda()
        xb = codec._as_bytes_view(x)
        dt = codec.codec_dtype(dtype)
        scratch = torch.empty(L.lz_codec_scratch_bytes(n, dt), dtype=torch.uint8, device="cuda")
        cap = L.lz_codec_max_bytes(n, dt)
        out = torch.empty(cap, dtype=torch.uint8, device="cuda")
        total = torch.zeros(1, dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        dec = torch.empty_like(xb)
        s = torch.cuda.current_stream().cuda_stream

        def enc():
            L.lz_codec_encode(xb.data_ptr(), n, codec.with_level(dt, level), scratch.data_ptr(), scratch.numel(), out.data_ptr(),
                              cap, total.data_ptr(), nblocks, s)

        def dcd():
            L.lz_codec_decode(out.data_ptr(), cap, dec.data_ptr(), n, dt, status.data_ptr(), nblocks, s)

        t_enc = _time(enc, iters, warmup, flush)
        t_dec = _time(dcd, iters, warmup, flush)
        torch.cuda.synchronize()
        ok = int(status.item()) == 0 and torch.equal(dec.view(torch.uint8), xb.view(torch.uint8))
        cb = int(total.item())
        rows.append({
            "Data size": csvfmt.size_label(nbytes),
            "size_bytes": nbytes,
            "comp_time_ms": round(t_enc, 4),
            "decomp_time_ms": round(t_dec, 4),
            "comp_throughput_gb_s": round(nbytes / t_enc / 1e6, 2),
            "decomp_throughput_gb_s": round(nbytes / t_dec / 1e6, 2),
            "compressed_bytes": cb,
            "compression_ratio": round(cb / nbytes, 4),
            "lossless": ok,
        })
        del x, scratch, out, dec
        torch.cuda.empty_cache()
    return rows


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--sizes-mb", default="4,16,64,128,256,1024")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--dist", default="normal", choices=["normal", "activation"])
    ap.add_argument("--std", type=float, default=0.02)
    ap.add_argument("--nblocks", type=int, default=0)
    ap.add_argument("--level", default="ans", choices=sorted(codec.LEVELS))
    ap.add_argument("--csv", default=None)
    a = ap.parse_args()
    dtype = getattr(torch, a.dtype)
    rows = run([int(s) for s in a.sizes_mb.split(",")], dtype, a.iters, a.warmup, a.dist, a.std, a.nblocks,
               a.level)
    for r in rows:
        print(r, flush=True)
    if a.csv:
        csvfmt.write_rows(a.csv, csvfmt.SCHEMA_D, rows)
        csvfmt.write_sidecar(a.csv, {"bench": "codec", "dtype": a.dtype, "dist": a.dist, "std": a.std,
                                     "level": a.level,
                                     "timing": "CUDA events, median of iters"})


if __name__ == "__main__":
    main()
