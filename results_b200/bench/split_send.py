"""Point-to-point send bench: rank 0 -> rank 1, raw vs split+rANS (schema B).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m results_b200.bench.split_send \
        --modes raw,split,nccl --dtype bfloat16 --csv out.csv [--sm-budget 16] [--chunk-mb 128]

B200 counterpart of the reference's UCCL-P2P benchmark
(uccl/p2p/benchmarks/benchmark_uccl_collective.py, named at raw/a.txt:590; result
files raw/result_bf16_split_rank0.csv, csv/p2p_split_send_vs_2baseline.csv):
sizes 256 B - 1 GB, modes "split" (split+rANS, LZip-P2P split_send), "pack"
(split + the codec's PACK level: table codes, faster than rANS), "raw"
(uncompressed native push) and "nccl" (send/recv baseline). Sweeps of dtype
(bf16/fp16/fp32/e4m3/e5m2), SM budget (green contexts) and chunking
(--chunk-mb: the transfer of one size is cut into chunks sent back to back,
bounding the staging memory) mirror the reference's figures. Throughput =
uncompressed bytes / device time (max over the two ranks).
"""
from __future__ import annotations

import argparse
import datetime
import os

import torch
import torch.distributed as dist

from ..utils import csvfmt


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--modes", default="raw,split,nccl",
                    help="raw, split (split+rANS), pack (split + PACK table codes), nccl, direct (zero copy "
                         "into a symmetric receive buffer), ce (the same by copy-engine DMA)")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--min-bytes", type=int, default=256)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--sm-budget", type=int, default=0)
    ap.add_argument("--chunk-mb", type=int, default=0)
    ap.add_argument("--std", type=float, default=0.02)
    ap.add_argument("--csv", default=None)
    return ap.parse_args()


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
    from results_b200.parallel import weights
    from results_b200.utils.sm_budget import SmBudget

    direct = bool({"direct", "ce"} & set(a.modes.split(",")))
    if direct and world != 2:
        raise SystemExit("modes 'direct' and 'ce' (zero copy into a symmetric receive buffer) run on exactly 2 ranks")
    comm = lz.init(config=Config(user_bytes=(a.max_bytes + 64 * MiB) if direct else 16 * MiB,
                                 stage_bytes=512 * MiB, timeout_s=60.0))
    dtype = getattr(torch, a.dtype)
    es = torch.empty((), dtype=dtype).element_size()
    budget = SmBudget(local, a.sm_budget) if a.sm_budget else None
    nblocks = min(3 * (budget.sm_count if budget else comm.sm_count), 512)
    engines = {"raw": weights.WeightTransfer(comm, mode="raw", nblocks=nblocks),
               "split": weights.WeightTransfer(comm, mode="split_ans", nblocks=nblocks),
               "pack": weights.WeightTransfer(comm, mode="split_pack", nblocks=nblocks)}
    rows = []
    size = a.min_bytes
    sizes = []
    while size <= a.max_bytes:
        sizes.append(size)
        size *= 4 if size < (1 << 20) else 2
    stream = budget.stream if budget else torch.cuda.current_stream()
    for nbytes in sizes:
        n = max(nbytes // es, 2)
        g = torch.Generator(device="cuda").manual_seed(5)
        x = (torch.randn(n, device="cuda", generator=g) * a.std).to(dtype)
        if rank != 0:
            x = torch.empty_like(x)
        chunk = (a.chunk_mb * MiB // es) if a.chunk_mb else n
        parts = [x[i:i + chunk] for i in range(0, n, chunk)]
        if direct:
            comm.reset_alloc()
            sym = comm.empty(n, dtype)
            sym_parts = [sym[i:i + chunk] for i in range(0, n, chunk)]
        for mode in a.modes.split(","):
            def once():
                if mode == "nccl":
                    for p in parts:
                        if rank == 0:
                            dist.send(p, 1)
                        elif rank == 1:
                            dist.recv(p, 0)
                elif mode == "direct":
                    engines["raw"].broadcast_direct(sym_parts, 0, src_tensors=parts if rank == 0 else None,
                                                    relay=False, copy_engine=False)
                elif mode == "ce":
                    engines["raw"].send_copy_engine(sym_parts, 0, 1, src_tensors=parts if rank == 0 else None)
                else:
                    eng = engines[mode]
                    for p in parts:
                        if rank == 0:
                            eng.send([p], 1)
                        elif rank == 1:
                            eng.recv([p], 0)
            with torch.cuda.stream(stream):
                for _ in range(a.warmup):
                    once()
                stream.synchronize()
                dist.barrier(group=ctrl)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(a.iters):
                    once()
                e1.record(stream)
                stream.synchronize()
            ms = e0.elapsed_time(e1) / a.iters
            t = torch.tensor([ms], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctrl)
            ms = float(t.item())
            comm.check()
            gbs = nbytes / (ms * 1e-3) / 1e9
            if rank == 0:
                rows.append({"role": "Client", "size_bytes": nbytes, "size_pretty": csvfmt.size_label(nbytes),
                             "gbps": round(gbs * 8, 4), "gb_sec": round(gbs, 4), "mode": mode})
                print(f"{mode:>6} {csvfmt.size_label(nbytes):>8}: {gbs:8.2f} GB/s", flush=True)
    if rank == 0 and a.csv:
        csvfmt.write_rows(a.csv, csvfmt.SCHEMA_B + ["mode"], rows)
        csvfmt.write_sidecar(a.csv, {"bench": "split_send", "dtype": a.dtype, "sm_budget": a.sm_budget,
                                     "chunk_mb": a.chunk_mb, "timing": "CUDA events, max over ranks"})
    if budget:
        budget.close()
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
