#!/usr/bin/env python
"""Headline benchmark: bf16 sum-allreduce bus bandwidth, 1 GiB per rank.

The headline metric ("allreduce bus GB/s vs size @2/4/8 GPU") at
the reference's headline message size (1 GB, csv/single_node_allreduce.csv:7
and csv/allreduce_throughput.csv:8 of the reference). One rank per GPU.

    python bench.py --gpus 1 --steps 50 --warmup 5
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...
    python bench.py --impl reference   # the reference's own arm
    python bench.py --impl nccl        # NCCL all_reduce through the same harness

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the
launching stream; the reported time is the max over ranks. Inputs are 1 GiB
per rank (> 126 MB L2), so no L2 flush is needed between steps.
"value" is the whole-job aggregate: sum over ranks of the per-rank bus
bandwidth busbw = algbw * 2(N-1)/N (for N = 1 the bus factor is taken as 1:
a one-rank allreduce is one read+write pass of the buffer).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import socket
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REF_BUSBW_1GB_WS8 = 53.60  # LZip two-shot, 1 GB, ws=8 (reference S/compression.csv:8)
# The reference's published 1 GB results as whole-job aggregates (busbw per
# rank x ranks), the same unit as "value": ws=2 LZip two-shot 54.68 GB/s algbw
# = busbw (csv/allreduce_throughput.csv:8); ws=8 53.60 GB/s busbw per rank.
REF_AGGREGATE_1GB = {2: 54.68 * 2, 8: REF_BUSBW_1GB_WS8 * 8}
METRIC = "allreduce_bus_GBps"


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "nccl"], default="ours")
    ap.add_argument("--size-mb", type=int, default=1024, help="MiB per rank")
    ap.add_argument("--algo", default="auto")
    ap.add_argument("--dtype", default="bfloat16", choices=["bfloat16", "float16", "float32"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-check", action="store_true")
    return ap.parse_args()


def _setup(args):
    import torch
    import torch.distributed as dist

    if "WORLD_SIZE" not in os.environ:
        os.environ.update({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0",
                           "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port())})
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=180))
    ctrl = dist.new_group(backend="gloo")
    return rank, world, local, ctrl


def _max_over_ranks(v: float, ctrl) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctrl)
    return float(t.item())


def _timed(step, steps, warmup, ctrl, devices):
    import torch
    import torch.distributed as dist

    from results_b200.utils.clocks import ClockSampler

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier(group=ctrl)
    sampler = ClockSampler(devices).start()
    s = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    dist.barrier(group=ctrl)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(steps):
        step()
    e1.record(s)
    torch.cuda.synchronize()
    dist.barrier(group=ctrl)
    sampler.stop()
    ms = e0.elapsed_time(e1) / steps
    return _max_over_ranks(ms, ctrl), sampler.summary()


def main():
    args = parse()
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    rank_env = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank_env == 0:
            print(json.dumps({
                "impl": "reference",
                "unavailable": "the reference (monopodium/results) is not pip-installable: no setup.py "
                               "or pyproject.toml, so baseline/_ref could not be installed offline",
                "metric": METRIC, "n_gpus": world_env}))
        return 0

    import torch
    import torch.distributed as dist

    rank, world, local, ctrl = _setup(args)
    dtype = getattr(torch, args.dtype)
    esize = torch.empty((), dtype=dtype).element_size()
    nbytes = args.size_mb << 20
    n = nbytes // esize
    bus = 2.0 * (world - 1) / world if world > 1 else 1.0

    def bw(ms):
        algbw = nbytes / (ms * 1e-3) / 1e9
        return algbw, algbw * bus

    comm = None
    launches_per_step = 0
    if args.impl == "ours":
        import results_b200 as lz
        from results_b200.config import Config, MiB

        cfg = Config(user_bytes=3 * nbytes + 64 * MiB, stage_bytes=64 * MiB, oneshot_bytes=8 * MiB)
        comm = lz.init(config=cfg)
        x = comm.empty(n, dtype)
        y = comm.empty(n, dtype)
        g = torch.Generator(device="cuda").manual_seed(1234 + rank)
        x.copy_((torch.randn(n, device="cuda", generator=g) * 1e-2).to(dtype))
        algo = args.algo
        if algo == "auto":
            algo = lz.select_algo(nbytes, world, comm.has_multicast, True)

        def step():
            comm.allreduce_(x, y, algo=algo)

        launches_per_step = 1
    else:
        algo = "nccl"
        x = (torch.randn(n, device="cuda") * 1e-2).to(dtype)

        def step():
            dist.all_reduce(x)

    ms, clocks = _timed(step, args.steps, args.warmup, ctrl, [local])
    if comm is not None:
        comm.check()
    algbw, busbw = bw(ms)

    check = None
    if args.impl == "ours" and not args.no_check:
        m = 1 << 16
        acc = torch.zeros(m, device="cuda", dtype=torch.float32)
        for r in range(world):
            g = torch.Generator(device="cuda").manual_seed(1234 + r)
            acc += (torch.randn(n, device="cuda", generator=g)[:m] * 1e-2).to(dtype).float()
        got = y[:m].float()
        err = ((got - acc).abs().max() / acc.abs().max()).item()
        check = {"max_rel_err_first_64k": err, "bitexact": bool(torch.equal(y[:m], acc.to(dtype)))}

    e2e = None
    if not args.no_e2e:
        # End to end through the public API: H2D of this step's input from
        # pinned host memory, the allreduce, D2H of a 4 KiB slice of the result.
        host_in = torch.empty(n, dtype=dtype, pin_memory=True)
        host_in.copy_(x.cpu() if args.impl == "nccl" else torch.zeros(n, dtype=dtype))
        host_out = torch.empty(4096 // esize, dtype=dtype, pin_memory=True)
        if args.impl == "ours":
            import results_b200 as lz

            xin = [x, comm.empty(n, dtype)]
            copy_s = torch.cuda.Stream()
            ready = [torch.cuda.Event(), torch.cuda.Event()]
            consumed = [torch.cuda.Event(), torch.cuda.Event()]
            state = {"k": 0}

            def e2e_step():
                k = state["k"]
                buf = xin[k % 2]
                with torch.cuda.stream(copy_s):
                    if k >= 2:
                        copy_s.wait_event(consumed[k % 2])
                    buf.copy_(host_in, non_blocking=True)
                    ready[k % 2].record(copy_s)
                cs = torch.cuda.current_stream()
                cs.wait_event(ready[k % 2])
                lz.allreduce(buf, algo=algo, out=y, comm=comm)
                consumed[k % 2].record(cs)
                host_out.copy_(y[: host_out.numel()], non_blocking=True)
                state["k"] = k + 1
        else:  # the same double-buffered pipeline around NCCL
            xin = [x, torch.empty_like(x)]
            copy_s = torch.cuda.Stream()
            ready = [torch.cuda.Event(), torch.cuda.Event()]
            consumed = [torch.cuda.Event(), torch.cuda.Event()]
            state = {"k": 0}

            def e2e_step():
                k = state["k"]
                buf = xin[k % 2]
                with torch.cuda.stream(copy_s):
                    if k >= 2:
                        copy_s.wait_event(consumed[k % 2])
                    buf.copy_(host_in, non_blocking=True)
                    ready[k % 2].record(copy_s)
                cs = torch.cuda.current_stream()
                cs.wait_event(ready[k % 2])
                dist.all_reduce(buf)
                consumed[k % 2].record(cs)
                host_out.copy_(buf[: host_out.numel()], non_blocking=True)
                state["k"] = k + 1

        e_ms, _ = _timed(e2e_step, args.steps, args.warmup, ctrl, [local])
        _, e_bus = bw(e_ms)
        e2e = {"value": round(world * e_bus, 3), "unit": "GB/s", "ms_per_step": round(e_ms, 4),
               "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": host_out.numel() * esize,
               "api": "results_b200.allreduce" if args.impl == "ours" else "torch.distributed.all_reduce"}

    if rank == 0:
        value = world * busbw
        out = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / REF_AGGREGATE_1GB[world], 3) if world in REF_AGGREGATE_1GB else None,
            "dtype": {"bfloat16": "bf16", "float16": "fp16", "float32": "fp32"}[args.dtype],
            "data": "synthetic: N(0, 1e-2) per rank from a fixed seed",
            "impl": args.impl,
            "config": {
                "model": f"allreduce sum {args.dtype} {args.size_mb} MiB per rank",
                "global_batch": world,
                "seq_len": n,
                "parallelism": f"dp{world}",
                "algo": algo,
                "bytes_per_rank": nbytes,
                "busbw_GBps_per_rank": round(busbw, 3),
                "algbw_GBps": round(algbw, 3),
                "bus_factor": bus,
                "l2": "1 GiB inputs per rank exceed the 126 MB L2; no flush between steps",
                "timing": "CUDA events on the launching stream, max over ranks",
                "baseline_ref": ("reference LZip two-shot at 1 GB as a whole-job aggregate: ws=2 109.36 GB/s, "
                                 "ws=8 428.8 GB/s (53.60 busbw per rank); H200 + EFA; none published for 1 or 4"),
            },
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
        }
        if comm is not None:
            out["config"]["multicast"] = comm.has_multicast
        if check is not None:
            out["check"] = check
        print(json.dumps(out), flush=True)
    if comm is not None:
        import results_b200 as lz

        lz.shutdown()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
