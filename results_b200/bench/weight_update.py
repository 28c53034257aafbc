"""RL weight-update bench: trainer rank 0 -> inference ranks 1..N-1.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m results_b200.bench.weight_update \
        --model glm4-9b --modes ours_raw,ours_split,nccl_bcast,nccl_send --csv out.csv

Modes
  ours_raw     native transfer, raw bytes (NVLS multimem broadcast when every rank receives)
  ours_split   native transfer, split+rANS encoded (bit-exact), same paths
  ours_pack    native transfer, split + the codec's PACK level (table codes), same paths
  ours_p2p     native point-to-point transfer to each receiver in turn (split+rANS)
  ours_direct  native zero-copy raw broadcast into receivers' symmetric weight tensors
               (relay broadcast with multimem.st forwarding for more than 2 ranks)
  ours_ce      copy-engine DMA into each receiver's symmetric weights (no SM moves data)
  ours_staged  raw broadcast into the receivers' ordinary (non-symmetric) weight tensors:
               relay broadcast (copy engines at 2 ranks) into double-buffered symmetric
               staging, copied out on a side stream while the next bucket moves
  nccl_bcast   per-tensor torch.distributed.broadcast, the reference's update path
               (back_up/update_weight_from_distributed.py:422-449)
  nccl_send    per-tensor send from rank 0 to every receiver (batched isend/irecv)

Reports the whole-model update time (device time, max over ranks) and, with
--per-tensor, schema-B' rows per distinct tensor shape like the reference's
raw/GLM9B-0414_split_rank0.csv. Receivers verify every tensor bit-exactly
against the sender through per-tensor checksums.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from ..utils import csvfmt


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="glm4-9b")
    ap.add_argument("--layers", type=int, default=0, help="override layer count (0: the model's)")
    ap.add_argument("--modes", default="ours_raw,ours_split,nccl_bcast,nccl_send")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--bucket-mb", type=int, default=1024)
    ap.add_argument("--stage-mb", type=int, default=256, help="staging buffer size of ours_staged (two of them)")
    ap.add_argument("--encode-fraction", type=float, default=1.0)
    ap.add_argument("--per-tensor", action="store_true")
    ap.add_argument("--per-tensor-iters", type=int, default=20)
    ap.add_argument("--csv", default=None)
    ap.add_argument("--json", default=None)
    return ap.parse_args()


def _max(v, ctrl):
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctrl)
    return float(t.item())


def checksum(t: torch.Tensor) -> int:
    v = t.view(-1).view(torch.int16 if t.element_size() == 2 else torch.int32).to(torch.int64)
    w = torch.arange(1, v.numel() + 1, device=t.device, dtype=torch.int64) % 65521
    return int((v * w).sum().item())


def main():
    a = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=600))
    ctrl = dist.new_group(backend="gloo")
    import results_b200 as lz
    from results_b200.config import Config, MiB
    from results_b200.models import shapes
    from results_b200.parallel import weights

    fn = shapes.MODELS[a.model]
    specs = fn(layers=a.layers) if a.layers else fn()
    total_bytes = shapes.total_params(specs) * 2
    direct = bool({"ours_direct", "ours_ce"} & set(a.modes.split(",")))
    user = (total_bytes + 256 * MiB) if direct else 64 * MiB
    if "ours_staged" in a.modes.split(","):
        user += 2 * a.stage_mb * MiB + 64 * MiB
    comm = lz.init(config=Config(user_bytes=user, stage_bytes=512 * MiB, timeout_s=60.0))
    sd = shapes.make_state_dict(specs, seed=1, empty=(rank != 0))
    names = list(sd.keys())
    tensors = list(sd.values())
    sym = [comm.empty(t.shape, t.dtype) for t in tensors] if direct else None  # collective, same offsets
    sym_of = {id(t): d for t, d in zip(tensors, sym)} if direct else {}
    bucket = a.bucket_mb * MiB
    engines = {
        "ours_raw": weights.WeightTransfer(comm, mode="raw"),
        "ours_split": weights.WeightTransfer(comm, mode="split_ans", encode_fraction=a.encode_fraction),
        "ours_pack": weights.WeightTransfer(comm, mode="split_pack", encode_fraction=a.encode_fraction),
        "ours_p2p": weights.WeightTransfer(comm, mode="split_ans", encode_fraction=a.encode_fraction),
    }

    def run(mode, ts):
        if mode == "ours_staged":
            engines["ours_raw"].broadcast_staged(ts, 0, stage_bytes=a.stage_mb * MiB)
            return
        if mode == "ours_direct":
            dst = [sym_of[id(t)] for t in ts]
            engines["ours_raw"].broadcast_direct(dst, 0, src_tensors=ts if rank == 0 else None)
            return
        if mode == "ours_ce":  # copy-engine DMA into each receiver's symmetric weights, one after another
            dst = [sym_of[id(t)] for t in ts]
            for d in range(1, world):
                engines["ours_raw"].send_copy_engine(dst, 0, d, src_tensors=ts if rank == 0 else None)
            return
        if mode in ("ours_raw", "ours_split", "ours_pack"):
            eng = engines[mode]
            for bkt in weights.buckets(list(zip(range(len(ts)), ts)), bucket):
                eng.broadcast([t for _, t in bkt], 0)
        elif mode == "ours_p2p":
            eng = engines[mode]
            for bkt in weights.buckets(list(zip(range(len(ts)), ts)), bucket):
                bt = [t for _, t in bkt]
                if rank == 0:
                    for d in range(1, world):
                        eng.send(bt, d)
                else:
                    eng.recv(bt, 0)
        elif mode == "nccl_bcast":
            works = [dist.broadcast(t, src=0, async_op=True) for t in ts]
            for w in works:
                w.wait()
        elif mode == "nccl_send":
            for t in ts:
                ops = []
                if rank == 0:
                    ops = [dist.P2POp(dist.isend, t, d) for d in range(1, world)]
                else:
                    ops = [dist.P2POp(dist.irecv, t, 0)]
                for w in dist.batch_isend_irecv(ops):
                    w.wait()

    results = {}
    ref_sums = None
    if a.modes:
        sums = [checksum(t) for t in tensors] if rank == 0 else None
        obj = [sums]
        dist.broadcast_object_list(obj, src=0, group=ctrl)
        ref_sums = obj[0]
    for mode in a.modes.split(","):
        if world == 1:
            break
        if rank != 0:
            for t in (sym if mode in ("ours_direct", "ours_ce") else tensors):
                t.fill_(0)
        for _ in range(a.warmup):
            run(mode, tensors)
        torch.cuda.synchronize()
        dist.barrier(group=ctrl)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(a.iters):
            run(mode, tensors)
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / a.iters
        sec = _max(e0.elapsed_time(e1) / a.iters / 1e3, ctrl)
        wall = _max(wall, ctrl)
        comm.check()
        ok = True
        if rank != 0:
            got = sym if mode in ("ours_direct", "ours_ce") else tensors
            ok = all(checksum(t) == s for t, s in zip(got, ref_sums))
        okt = torch.tensor([0 if ok else 1])
        dist.all_reduce(okt, group=ctrl)
        results[mode] = {"sec": sec, "wall_sec": wall, "bitexact": int(okt.item()) == 0,
                         "GBps_per_receiver": total_bytes / sec / 1e9}
        if rank == 0:
            print(f"{mode:>10}: {sec:.4f} s/update ({total_bytes / sec / 1e9:.1f} GB/s per receiver), "
                  f"bitexact={results[mode]['bitexact']}", flush=True)

    rows = []
    if a.per_tensor and world > 1:
        seen = {}
        for nm, t in zip(names, tensors):
            key = nm.split(".")[-2] if nm.count(".") > 1 else nm
            if key not in seen and t.numel() * t.element_size() >= (16 << 20):
                seen[key] = (nm, t)
        for key, (nm, t) in seen.items():
            for mode in a.modes.split(","):
                for _ in range(2):
                    run(mode, [t])
                torch.cuda.synchronize()
                dist.barrier(group=ctrl)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(a.per_tensor_iters):
                    run(mode, [t])
                e1.record()
                torch.cuda.synchronize()
                sec = _max(e0.elapsed_time(e1) / a.per_tensor_iters / 1e3, ctrl)
                nb = t.numel() * t.element_size()
                if rank == 0:
                    rows.append({"role": "Client", "mode": mode, "size_bytes": nb,
                                 "size_pretty": f"{nb / (1 << 20):.1f} MB", "gbps": round(nb * 8 / sec / 1e9, 4),
                                 "gb_sec": round(nb / sec / 1e9, 4), "iters": a.per_tensor_iters, "rank": 0,
                                 "world_size": world, "tensor": key})
    if rank == 0:
        summary = {"model": a.model, "params": shapes.total_params(specs), "bytes": total_bytes, "world": world,
                   "multicast": comm.has_multicast, "results": results}
        if "nccl_send" in results:
            for m in ("ours_raw", "ours_split", "ours_pack", "ours_direct", "ours_ce", "ours_staged"):
                if m in results:
                    summary[f"speedup_{m}_vs_nccl_send"] = results["nccl_send"]["sec"] / results[m]["sec"]
        if "nccl_bcast" in results:
            for m in ("ours_raw", "ours_split", "ours_pack", "ours_direct", "ours_ce", "ours_staged"):
                if m in results:
                    summary[f"speedup_{m}_vs_nccl_bcast"] = results["nccl_bcast"]["sec"] / results[m]["sec"]
        print(json.dumps(summary), flush=True)
        if a.json:
            with open(a.json, "w") as f:
                json.dump(summary, f, indent=1)
        if a.csv and rows:
            csvfmt.write_rows(a.csv, csvfmt.SCHEMA_B2, rows)
            csvfmt.write_sidecar(a.csv, {"bench": "weight_update", **summary})
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
