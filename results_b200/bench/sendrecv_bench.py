"""Blocking NCCL send/recv bench between two ranks (schema C), plus the
native point-to-point push for comparison.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m results_b200.bench.sendrecv_bench --csv out.csv

Counterpart of back_up/nccl_send_recv_bench.py:8-97 of the reference (fp32,
1 MB - 1 GB, CSV header data_size_MB,latency_sec,throughput_GBps). The
reference timed with the wall clock on rank 0; here device time with CUDA
events, max over ranks, is reported (wall time also recorded).
"""
from __future__ import annotations

import argparse
import datetime
import os
import time

import torch
import torch.distributed as dist

from ..utils import csvfmt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="1,2,4,8,16,32,64,128,256,512,1024")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--native", action="store_true", help="also time the native raw push")
    ap.add_argument("--csv", default=None)
    a = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=300))
    ctrl = dist.new_group(backend="gloo")
    eng = None
    if a.native:
        import results_b200 as lz
        from results_b200.config import Config, MiB
        from results_b200.parallel import weights

        eng = weights.WeightTransfer(lz.init(config=Config(user_bytes=16 * MiB, stage_bytes=512 * MiB)),
                                     mode="raw")
    rows = []
    for mb in [int(s) for s in a.sizes_mb.split(",")]:
        t = torch.ones(mb * (1 << 20) // 4, dtype=torch.float32, device="cuda")
        for kind in (["nccl", "native"] if eng else ["nccl"]):
            def once():
                if kind == "nccl":
                    if rank == 0:
                        dist.send(t, 1)
                    elif rank == 1:
                        dist.recv(t, 0)
                else:
                    if rank == 0:
                        eng.send([t], 1)
                    elif rank == 1:
                        eng.recv([t], 0)
            for _ in range(3):
                once()
            torch.cuda.synchronize()
            dist.barrier(group=ctrl)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            w0 = time.perf_counter()
            e0.record()
            for _ in range(a.iters):
                once()
            e1.record()
            torch.cuda.synchronize()
            wall = (time.perf_counter() - w0) / a.iters
            sec = e0.elapsed_time(e1) / a.iters / 1e3
            m = torch.tensor([sec, wall], dtype=torch.float64)
            dist.all_reduce(m, op=dist.ReduceOp.MAX, group=ctrl)
            sec, wall = m.tolist()
            if rank == 0:
                rows.append({"data_size_MB": mb, "latency_sec": round(sec, 6),
                             "throughput_GBps": round(mb * (1 << 20) / sec / 1e9, 3), "kind": kind,
                             "wall_sec": round(wall, 6)})
                print(rows[-1], flush=True)
    if rank == 0 and a.csv:
        csvfmt.write_rows(a.csv, csvfmt.SCHEMA_C + ["kind", "wall_sec"], rows)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
