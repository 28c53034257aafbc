"""Lossless compressed allreduce sweep: data distribution x size x SM budget x
chunk size, against NCCL, with measured compression ratio and peak extra
device memory; plus the fp8 (e4m3 / e5m2) pair-packed compressed send of the
same tensors.

    torchrun --nproc-per-node 8 -m results_b200.bench.compressed_sweep --csv cz.csv
    torchrun --nproc-per-node 8 -m results_b200.bench.compressed_sweep \
        --dists grad,act --sizes-mb 4,64,256,1024 --sm-budgets 16,32,64,96,128,0 --chunks-mb 0,64,128,256

Distributions: ``grad`` = N(0, 1e-3) (gradient-like); ``act`` = N(0, 1) with 1 %
of the elements multiplied by 50 (activation-like with outliers); per rank
from a fixed seed. SM budgets use CUDA green contexts (0 = whole GPU); the
kernel grid is sized to what the budget keeps resident. ``--chunks-mb``
processes the tensor in chunks of that size inside the one launch (a ring of
two chunks' slots bounds the stage memory; 0 = one chunk). ``extra_mem_bytes``
is the stage the native kernel needs for the call plus any torch allocations
made by the call (NCCL: 0).
The fp8 rows cast the tensor to e4m3fn / e5m2, and rank 0 sends it through the
split+rANS transfer kernel (pair containers) to rank 1.

Reference counterparts: the compressed two-shot sweeps of
single_node_nccl_allreduce_benchmark/benchmark_both.py:350-690 (schema A) and
the UCCL SM-budget logs (raw/bf16_split_sm16_split_encode_time_count.txt,
raw/bf16_split_sm100_split_encode_time_count.txt).
"""
from __future__ import annotations

import argparse
import datetime
import os

import torch
import torch.distributed as dist

from ..utils import csvfmt

HEADER = ["dist", "dtype", "size_bytes", "size_label", "world_size", "sm_budget", "chunk_mb", "variant", "ms",
          "algbw_GBps", "busbw_GBps", "comp_ratio", "extra_mem_bytes", "exact"]


def _data(n: int, kind: str, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    if kind == "grad":
        return (torch.randn(n, device="cuda", generator=g) * 1e-3).to(torch.bfloat16)
    x = torch.randn(n, device="cuda", generator=g)
    mask = torch.rand(n, device="cuda", generator=g) < 0.01
    x[mask] *= 50.0
    return x.to(torch.bfloat16)


def _max(v: float, group) -> float:
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--dists", default="grad,act")
    ap.add_argument("--sizes-mb", default="4,64,256,1024")
    ap.add_argument("--sm-budgets", default="16,32,64,0")
    ap.add_argument("--chunks-mb", default="0,64,128,256")
    ap.add_argument("--variants", default="compressed,hybrid,compressed_pack,hybrid_pack",
                    help="compressed: reduce-scatter and all-gather compressed; hybrid: raw reduce-scatter, "
                         "compressed all-gather; the _pack suffix codes records with the codec's PACK "
                         "level (table codes) instead of rANS; a trailing _local encodes reduce-scatter "
                         "records locally and pushes them")
    ap.add_argument("--fp8", action="store_true", default=True)
    ap.add_argument("--no-fp8", dest="fp8", action="store_false")
    ap.add_argument("--trace", action="store_true",
                    help="after timing, run the call again with the kernel's per-CTA phase tracer and print "
                         "the mean microseconds per phase (rank 0)")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--csv", default=None)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()),
                            timeout=datetime.timedelta(seconds=600))
    ctrl = dist.new_group(backend="gloo")
    import results_b200 as lz
    from results_b200.config import Config, MiB
    from results_b200.ops import codec
    from results_b200.parallel import compressed as cz
    from results_b200.parallel import weights
    from results_b200.utils.sm_budget import SmBudget

    sizes = [int(s) * MiB for s in a.sizes_mb.split(",")]
    budgets = [int(s) for s in a.sm_budgets.split(",")]
    chunks = [int(s) for s in a.chunks_mb.split(",")]
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    stage = cz.stage_bytes_needed(max(sizes) // 2, torch.bfloat16, world, 3 * sms) + 64 * MiB
    comm = lz.init(config=Config(user_bytes=64 * MiB, stage_bytes=stage, timeout_s=60.0))
    streams = {0: None}
    for b in budgets:
        if b:
            streams[b] = SmBudget(torch.cuda.current_device(), b)
    rows = []

    def timed(fn, stream):
        ctx = torch.cuda.stream(stream.stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream())
        with ctx:
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
        return _max(e0.elapsed_time(e1) / a.iters, ctrl)

    for kind in a.dists.split(","):
        for nbytes in sizes:
            n = nbytes // 2
            x = _data(n, kind, 900 + rank)
            ratios = {lv: _max(codec.compression_ratio(x, level=lv), ctrl) for lv in ("ans", "pack")}
            acc = torch.zeros(n, device="cuda")
            for r in range(world):  # the exact answer: fp32 sum in rank order, rounded once
                acc += _data(n, kind, 900 + r).float()
            ref = acc.to(torch.bfloat16)
            del acc
            y = torch.empty_like(x)
            base = dict(dist=kind, dtype="bfloat16", size_bytes=nbytes, size_label=csvfmt.size_label(nbytes),
                        world_size=world)
            busf = 2 * (world - 1) / world
            buf = x.clone()
            nccl_ms = ms = timed(lambda: dist.all_reduce(buf), None)
            rows.append({**base, "sm_budget": 0, "chunk_mb": 0, "variant": "nccl", "ms": round(ms, 4),
                         "algbw_GBps": round(nbytes / ms / 1e6, 2), "busbw_GBps": round(nbytes / ms / 1e6 * busf, 2),
                         "comp_ratio": "", "extra_mem_bytes": 0, "exact": ""})
            for b in budgets:
                st = streams[b]
                nb = 3 * (st.sm_count if st is not None else sms)
                for cmb, var in [(cm, vv) for cm in chunks for vv in a.variants.split(",")]:
                    if cmb and cmb * MiB >= nbytes:
                        continue
                    level = "pack" if "_pack" in var else "ans"
                    ratio = ratios[level]

                    def run(hybrid=var.startswith("hybrid"), level=level, cb=cmb * MiB, loc=var.endswith("_local")):
                        cz.compressed_allreduce(x, y, comm=comm, nblocks=nb, hybrid=hybrid, level=level,
                                                chunk_bytes=cb, stage_local=loc)

                    torch.cuda.reset_peak_memory_stats()
                    m0 = torch.cuda.memory_allocated()
                    ms = timed(run, st)
                    extra = cz.stage_bytes_needed(n, torch.bfloat16, world, nb, chunk_elems=cmb * MiB // 2) + \
                        (torch.cuda.max_memory_allocated() - m0)
                    if a.trace:
                        tbuf = cz.trace_buffer(comm, nb)
                        ctx = torch.cuda.stream(st.stream) if st is not None else torch.cuda.stream(
                            torch.cuda.current_stream())
                        with ctx:
                            for _ in range(a.iters):
                                cz.compressed_allreduce(x, y, comm=comm, nblocks=nb, hybrid=var.startswith("hybrid"),
                                                        level=level, chunk_bytes=cmb * MiB,
                                                        stage_local=var.endswith("_local"), trace=tbuf)
                        torch.cuda.synchronize()
                        if rank == 0:
                            print(f"trace {kind} {csvfmt.size_label(nbytes)} sm={b or sms} chunk={cmb}MB {var}: "
                                  f"{cz.summarize_trace(tbuf, a.iters)}", flush=True)
                    exact = bool(torch.equal(y, ref))
                    rows.append({**base, "sm_budget": b or sms, "chunk_mb": cmb, "variant": var,
                                 "ms": round(ms, 4), "algbw_GBps": round(nbytes / ms / 1e6, 2),
                                 "busbw_GBps": round(nbytes / ms / 1e6 * busf, 2), "comp_ratio": round(ratio, 4),
                                 "extra_mem_bytes": int(_max(extra, ctrl)), "exact": exact})
                    if rank == 0:
                        print(f"{kind} {csvfmt.size_label(nbytes):>7} sm={b or sms:3d} chunk={cmb:4d}MB "
                              f"{var} {ms:8.3f} ms ({nbytes / ms / 1e6 * busf:7.1f} busbw) "
                              f"nccl {nccl_ms:8.3f} ms ratio {ratio:.3f} "
                              f"exact={exact}", flush=True)
            if a.fp8 and world >= 2:
                eng = weights.WeightTransfer(comm, mode="split_ans")
                x0 = _data(n, kind, 900) if rank == 1 else x  # the sender's (rank 0's) tensor

                def cast(t, f8):
                    return t.float().clamp(-448, 448).to(f8) if f8 == torch.float8_e4m3fn else t.to(f8)

                for f8 in (torch.float8_e4m3fn, torch.float8_e5m2):
                    xf = cast(x, f8)
                    want = cast(x0, f8)
                    dst = torch.empty_like(xf) if rank == 1 else xf
                    fratio = _max(codec.compression_ratio(xf), ctrl)

                    def send():
                        if rank == 0:
                            eng.send([xf], 1)
                        elif rank == 1:
                            eng.recv([dst], 0)

                    ms = timed(send, None)
                    exact = bool(torch.equal(dst.view(torch.uint8), want.view(torch.uint8))) if rank == 1 else True
                    ok = torch.tensor([0 if exact else 1])
                    dist.all_reduce(ok, group=ctrl)
                    fb = xf.numel()
                    rows.append({**base, "dtype": str(f8).replace("torch.", ""), "size_bytes": fb,
                                 "size_label": csvfmt.size_label(fb), "sm_budget": sms, "chunk_mb": 0,
                                 "variant": "fp8_packed_send", "ms": round(ms, 4),
                                 "algbw_GBps": round(fb / ms / 1e6, 2), "busbw_GBps": "",
                                 "comp_ratio": round(fratio, 4), "extra_mem_bytes": 0,
                                 "exact": int(ok.item()) == 0})
                    if rank == 0:
                        print(f"{kind} {str(f8)} {csvfmt.size_label(fb):>7} packed send 0->1 {ms:8.3f} ms "
                              f"ratio {fratio:.3f} exact={int(ok.item()) == 0}", flush=True)
            del x, y, ref, buf
    for st in streams.values():
        if st is not None:
            st.close()
    if rank == 0 and a.csv:
        csvfmt.write_rows(a.csv, HEADER, rows)
        csvfmt.write_sidecar(a.csv, {"bench": "compressed_sweep", "world": world,
                                     "timing": "CUDA events on the (green-context) stream, max over ranks"})
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
