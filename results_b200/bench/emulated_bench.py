"""Single-GPU timing of the multi-rank kernel bodies through the R-rank emulator.

    python -m results_b200.bench.emulated_bench --world 8 --mb 256 --algos oneshot,twoshot,compressed
    (also: compressed_pack, hybrid_pack, ll, a2a_raw, a2a_compressed, relay, wx_raw, wx_split)

Every emulated rank's heap lives on one GPU and the collective runs as one
cooperative launch, so the numbers measure the kernel bodies (barriers,
partitioning, rank-order fp32 reduction, codec) against HBM instead of
NVLink. It is the workload for kernel profiles of the allreduce and
compressed-allreduce bodies, which cannot be captured on a multi-rank run.
Reported: device time per call and HBM bytes moved per call over that time
(each rank reads its input and all peers' shards, and writes its output).
"""
from __future__ import annotations

import argparse
import json

import torch

from results_b200.parallel.emulate import EmulatedWorld


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--mb", type=int, default=256, help="per-rank message size in MiB")
    ap.add_argument("--kb", type=int, default=0, help="per-rank message size in KiB (overrides --mb)")
    ap.add_argument("--algos", default="oneshot,twoshot,compressed")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--nblocks", type=int, default=0)
    args = ap.parse_args(argv)
    dt = getattr(torch, args.dtype)
    es = torch.empty((), dtype=dt).element_size()
    n = ((args.kb << 10) if args.kb else (args.mb << 20)) // es
    R = args.world
    oneshot = min(n * es, 8 << 20)
    stage = max(64 << 20, 2 * n * es + (96 << 20))
    heap = 2 * n * es + 2 * oneshot + stage + (16 << 20)
    w = EmulatedWorld(R, heap_bytes=heap, oneshot_bytes=oneshot, stage_bytes=stage)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ar_blocks = args.nblocks or max(1, sms // R)  # R grids of 512-thread CTAs stay co-resident
    ins = w.empty((n,), dt)
    outs = w.empty((n,), dt)
    g = torch.Generator(device="cuda").manual_seed(7)
    for r in range(R):
        ins[r].copy_(torch.randn(n, generator=g, device="cuda", dtype=torch.float32).mul_(0.02).to(dt))
    ref = torch.stack([t.float() for t in ins]).sum(0)
    rows = []
    for algo in args.algos.split(","):
        if algo == "oneshot" and n * es > oneshot:
            print(json.dumps({"algo": algo, "skipped": f"one-shot is limited to {oneshot} bytes"}), flush=True)
            continue
        if algo == "ll" and n * es > 256 * 1024:
            print(json.dumps({"algo": algo, "skipped": "ll is limited to 256 KB"}), flush=True)
            continue
        check = True
        if algo == "compressed":
            fn = lambda: w.compressed_allreduce(ins, outs, nblocks=args.nblocks)  # noqa: E731
        elif algo in ("compressed_pack", "hybrid_pack"):
            fn = lambda h=(algo == "hybrid_pack"): w.compressed_allreduce(  # noqa: E731
                ins, outs, nblocks=args.nblocks, hybrid=h, level="pack")
        elif algo in ("a2a_raw", "a2a_compressed"):
            fn = lambda c=(algo == "a2a_compressed"): w.all_to_all(ins, outs, compress=c,  # noqa: E731
                                                                   nblocks=args.nblocks)
            check = False
        elif algo == "relay":
            fn = lambda: w.broadcast_relay(0, [[o] for o in outs], [ins[0]], nblocks=ar_blocks)  # noqa: E731
            check = False
        elif algo in ("wx_raw", "wx_split"):
            fn = lambda e=(algo == "wx_split"): w.weight_transfer(  # noqa: E731
                0, list(range(1, R)), [[ins[0]]] + [[o] for o in outs[1:]], encode=e, nblocks=ar_blocks,
                broadcast_all=True)
            check = False
        else:
            fn = lambda a=algo: w.allreduce(ins, outs, algo=a, nblocks=ar_blocks)  # noqa: E731
        ms = _time(fn, args.iters, args.warmup)
        err = (outs[0].float() - ref).abs().max().item() if check else None
        # HBM bytes per rank of the emulated collective (every "peer" access
        # is local): one-shot = copy-in (2n) + R reads and one write of n;
        # two-shot = input read + push (2n) + reduce read n and 2n/R writes +
        # gather read and output write (2n(R-1)/R). The codec path has none.
        nb = n * es
        per_rank = {"oneshot": (R + 3) * nb, "twoshot": 3 * nb + 2 * nb / R + 2 * nb * (R - 1) / R}.get(algo)
        row = {"algo": algo, "world": R, "bytes_per_rank": nb, "ms": round(ms, 4),
               "hbm_GBps": round(R * per_rank / (ms * 1e-3) / 1e9, 1) if per_rank else None,
               "max_abs_err": err}
        rows.append(row)
        print(json.dumps(row), flush=True)
    w.close()
    return rows


if __name__ == "__main__":
    main()
