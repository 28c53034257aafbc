"""Prefill -> decode KV-cache transfer bench (P/D disaggregation).

    torchrun --nproc-per-node 2 -m results_b200.bench.kv_transfer --csv kv.csv

Rank 0 (prefill) sends the KV cache of one request, one K and one V tensor of
[tokens, kv_heads, head_dim] bf16 per layer, to rank 1 (decode). Token counts
and the output columns follow the reference's table
(csv/cccl_p2p_pd_disaggregation.csv: input tokens 7680 .. 102400, NCCL vs
compressed transfer latency in ms; its model is not recorded, so the KV shape
here is GLM-4-9B's: 40 layers, 2 KV heads of dim 128, 40 KB per token).

Modes: nccl (batched isend/irecv per tensor), ours_raw and ours_split (the
native point-to-point transfer kernel, raw or split+rANS encoded),
ours_direct (zero-copy SM stores into the receiver's symmetric KV buffers),
ours_ce (the same by copy-engine DMA).
Latency: CUDA events per rank around one whole request, max over ranks.
Data: N(0, 1) activations from a fixed seed; receivers are checked bit-exact.
"""
from __future__ import annotations

import argparse
import datetime
import os

import torch
import torch.distributed as dist

from ..utils import csvfmt

TOKENS = (7680, 10240, 15360, 25600, 51200, 76800, 102400)
HEADER = ["Input Token", "nccl kv cache transfer latency (ms)", "ours_raw latency (ms)",
          "ours_split latency (ms)", "ours_direct latency (ms)", "ours_ce latency (ms)", "kv_bytes", "bitexact"]


def _max(v: float, group) -> float:
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default=",".join(map(str, TOKENS)))
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--kv-heads", type=int, default=2)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--csv", default=None)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world != 2:
        print("runs on exactly 2 ranks (prefill -> decode)")
        return
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()),
                            timeout=datetime.timedelta(seconds=300))
    ctrl = dist.new_group(backend="gloo")
    import results_b200 as lz
    from results_b200.config import Config, MiB
    from results_b200.parallel import weights

    toks = [int(t) for t in a.tokens.split(",")]
    per_tok = 2 * a.layers * a.kv_heads * a.head_dim * 2
    max_bytes = max(toks) * per_tok
    comm = lz.init(config=Config(user_bytes=max_bytes + 256 * MiB, stage_bytes=512 * MiB, timeout_s=60.0))
    raw = weights.WeightTransfer(comm, mode="raw")
    split = weights.WeightTransfer(comm, mode="split_ans")
    rows = []
    for T in toks:
        shape = (T, a.kv_heads, a.head_dim)
        g = torch.Generator(device="cuda").manual_seed(T)
        src = [torch.randn(shape, device="cuda", generator=g).to(torch.bfloat16) for _ in range(2 * a.layers)]
        dst = [torch.empty_like(t) for t in src] if rank else src
        comm.reset_alloc()
        sym = [comm.empty(shape, torch.bfloat16) for _ in range(2 * a.layers)]

        def run(mode):
            if mode == "nccl":
                for t_s, t_d in zip(src, dst):
                    op = dist.P2POp(dist.isend, t_s, 1) if rank == 0 else dist.P2POp(dist.irecv, t_d, 0)
                    for w in dist.batch_isend_irecv([op]):
                        w.wait()
            elif mode == "ours_direct":
                raw.broadcast_direct(sym, 0, src_tensors=src if rank == 0 else None, relay=False, copy_engine=False)
            elif mode == "ours_ce":
                raw.send_copy_engine(sym, 0, 1, src_tensors=src if rank == 0 else None)
            else:
                eng = raw if mode == "ours_raw" else split
                if rank == 0:
                    eng.send(src, 1)
                else:
                    eng.recv(dst, 0)

        res, exact = {}, True
        for mode in ("nccl", "ours_raw", "ours_split", "ours_direct", "ours_ce"):
            if rank == 1:
                for t in (sym if mode in ("ours_direct", "ours_ce") else dst):
                    t.fill_(0)
            for _ in range(a.warmup):
                run(mode)
            torch.cuda.synchronize()
            dist.barrier(group=ctrl)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                run(mode)
            e1.record()
            torch.cuda.synchronize()
            comm.check()
            res[mode] = _max(e0.elapsed_time(e1) / a.iters, ctrl)
            if rank == 1:
                got = sym if mode in ("ours_direct", "ours_ce") else dst
                exact = exact and all(torch.equal(x.view(torch.int16), y.view(torch.int16))
                                      for x, y in zip(got, src))
        ok = torch.tensor([0 if exact else 1])
        dist.all_reduce(ok, group=ctrl)
        row = {"Input Token": T, "nccl kv cache transfer latency (ms)": round(res["nccl"], 3),
               "ours_raw latency (ms)": round(res["ours_raw"], 3),
               "ours_split latency (ms)": round(res["ours_split"], 3),
               "ours_direct latency (ms)": round(res["ours_direct"], 3),
               "ours_ce latency (ms)": round(res["ours_ce"], 3),
               "kv_bytes": T * per_tok, "bitexact": int(ok.item()) == 0}
        rows.append(row)
        if rank == 0:
            print(row, flush=True)
        del src, dst, sym
    if rank == 0 and a.csv:
        csvfmt.write_rows(a.csv, HEADER, rows)
        csvfmt.write_sidecar(a.csv, {"bench": "kv_transfer", "layers": a.layers, "kv_heads": a.kv_heads,
                                     "head_dim": a.head_dim, "timing": "CUDA events, max over ranks"})
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
