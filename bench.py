#!/usr/bin/env python
"""Headline benchmark: bf16 sum-allreduce bus bandwidth, 1 GiB per rank.

The headline metric ("allreduce bus GB/s vs size @2/4/8 GPU") at
the reference's headline message size (1 GB, csv/single_node_allreduce.csv:7
and csv/allreduce_throughput.csv:8 of the reference). One rank per GPU.

    python bench.py --gpus 1 --steps 50 --warmup 5
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...
    python bench.py --impl reference   # the reference's own NCCL benchmark code
    python bench.py --impl nccl        # NCCL all_reduce through this harness

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the
launching stream; the reported time is the max over ranks. Inputs are 1 GiB
per rank (> 126 MB L2), so no L2 flush is needed between steps.
"value" is the whole-job aggregate: sum over ranks of the per-rank bus
bandwidth busbw = algbw * 2(N-1)/N (for N = 1 the bus factor is taken as 1:
a one-rank allreduce is one read+write pass of the buffer).

Correctness: after timing, every rank rebuilds all ranks' inputs from their
seeds, sums them in fp32 in rank order, rounds once, and compares the whole
output tensor: the line reports mismatching elements and the largest distance
in units in the last place (ulp), max over ranks.

End to end ("e2e"): the same allreduce through the public API, each step
uploading that step's input from pinned host memory and reading the whole
result back into pinned host memory (both copies double-buffered on their own
streams, so the upload of step k+1 and the read-back of step k overlap the
collective).

The reference arm runs the reference's own code unchanged: ``bench_standard``
of single_node_nccl_allreduce_benchmark/benchmark_both.py:52-69 (the function
its main() uses for the NCCL column, bf16 uniform[-1, 1]; its timed loop
refills the tensor before every all_reduce, benchmark_both.py:61-66), imported
from ``baseline/_ref``. The fill-free fp32 loop of nccl_standard_allreduce.py:30-53
is reported beside it. That arm never imports this package.
"""
from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import os
import socket
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))

REF_BUSBW_1GB_WS8 = 53.60  # LZip two-shot, 1 GB, ws=8 (reference S/compression.csv:8)
# The reference's published 1 GB results as whole-job aggregates (busbw per
# rank x ranks), the same unit as "value": ws=2 LZip two-shot 54.68 GB/s algbw
# = busbw (csv/allreduce_throughput.csv:8); ws=8 53.60 GB/s busbw per rank.
REF_AGGREGATE_1GB = {2: 54.68 * 2, 8: REF_BUSBW_1GB_WS8 * 8}
METRIC = "allreduce_bus_GBps"
REF_SUBDIR = "single_node_nccl_allreduce_benchmark"


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
    ap.add_argument("--no-nccl-compare", action="store_true",
                    help="skip the NCCL all_reduce timed in the same harness beside ours")
    return ap.parse_args()


def _clock_sampler_cls():
    """NVML clock reader, loaded from its file so that the reference arm does
    not import the results_b200 package (only this read-only sampler)."""
    path = os.path.join(ROOT, "results_b200", "utils", "clocks.py")
    spec = importlib.util.spec_from_file_location("_bench_clocks", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.ClockSampler


def _env_defaults():
    if "WORLD_SIZE" not in os.environ:
        os.environ.update({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0",
                           "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port())})


def _setup(args):
    import torch
    import torch.distributed as dist

    _env_defaults()
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


def _timed(step, steps, warmup, ctrl, devices, finish=None):
    """W warm-up steps, then K steps between CUDA events on the current
    stream, bracketed by barrier + synchronize; returns (max ms, clocks).
    `finish` makes the current stream wait for side streams before the end
    event is recorded."""
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        step()
    if finish is not None:
        finish()
    torch.cuda.synchronize()
    dist.barrier(group=ctrl)
    sampler = _clock_sampler_cls()(devices).start()
    s = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    dist.barrier(group=ctrl)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(steps):
        step()
    if finish is not None:
        finish()
    e1.record(s)
    torch.cuda.synchronize()
    dist.barrier(group=ctrl)
    sampler.stop()
    ms = e0.elapsed_time(e1) / steps
    return _max_over_ranks(ms, ctrl), sampler.summary()


def _ordered_bits(t):
    """Float bit patterns mapped to integers whose difference counts ulps."""
    import torch

    if t.element_size() == 2:
        u = t.view(torch.int16).to(torch.int32)
        return torch.where(u < 0, -(u & 0x7FFF), u)
    u = t.view(torch.int32).to(torch.int64)
    return torch.where(u < 0, -(u & 0x7FFFFFFF), u)


def _input(rank, n, dtype):
    import torch

    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    return (torch.randn(n, device="cuda", generator=g) * 1e-2).to(dtype)


def _check_full(ys, world, n, dtype, ctrl):
    """Whole-tensor comparison of each output in `ys` (name -> tensor) against
    the fp32 rank-order sum of every rank's input, rounded once."""
    import torch

    acc = torch.zeros(n, device="cuda", dtype=torch.float32)
    for r in range(world):
        acc += _input(r, n, dtype).float()
    ref = acc.to(dtype)
    amax = float(acc.abs().max().item())
    out = {}
    for name, y in ys.items():
        y = y.view(-1)
        mism = int((y != ref).sum().item())
        err = float((y.float() - acc).abs().max().item()) / max(amax, 1e-30)
        ulp = int((_ordered_bits(y) - _ordered_bits(ref)).abs().max().item()) if y.element_size() == 2 else None
        mism = int(_max_over_ranks(float(mism), ctrl))
        err = _max_over_ranks(err, ctrl)
        rec = {"mismatch_elements": mism, "bitexact": mism == 0, "max_abs_err_over_max_abs": err}
        if ulp is not None:
            ulp = int(_max_over_ranks(float(ulp), ctrl))
            rec.update({"max_ulp": ulp, "within_1ulp": ulp <= 1})
        out[name] = rec
    del acc, ref
    torch.cuda.empty_cache()
    res = dict(out.pop("ours", {}))
    res.update({"elements_checked": n, "oracle": "fp32 sum of every rank's input in rank order, rounded once; "
                                                 "whole tensor, max over ranks"})
    if out:
        res["same_check_of"] = out
    return res


def _e2e(step_fn, host_in, host_out, dev_in, dev_out, steps, warmup, ctrl, local):
    """Double-buffered end-to-end loop: upload -> collective -> read-back."""
    import torch

    h2d = torch.cuda.Stream()
    d2h = torch.cuda.Stream()
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]
    produced = [torch.cuda.Event(), torch.cuda.Event()]
    drained = [torch.cuda.Event(), torch.cuda.Event()]
    state = {"k": 0}

    def one():
        k = state["k"]
        b = k % 2
        with torch.cuda.stream(h2d):
            if k >= 2:  # buffer b: step k-2 consumed it and (in place) read it back
                h2d.wait_event(consumed[b])
                h2d.wait_event(drained[b])
            dev_in[b].copy_(host_in[b], non_blocking=True)
            ready[b].record(h2d)
        cs = torch.cuda.current_stream()
        cs.wait_event(ready[b])
        if k >= 2:
            cs.wait_event(drained[b])
        step_fn(dev_in[b], dev_out[b])
        consumed[b].record(cs)
        produced[b].record(cs)
        with torch.cuda.stream(d2h):
            d2h.wait_event(produced[b])
            host_out[b].copy_(dev_out[b], non_blocking=True)
            drained[b].record(d2h)
        state["k"] = k + 1

    def finish():
        cs = torch.cuda.current_stream()
        cs.wait_stream(d2h)
        cs.wait_stream(h2d)

    return _timed(one, steps, warmup, ctrl, [local], finish=finish)


def _pinned_inputs(x, n, dtype):
    import torch

    host_in = [torch.empty(n, dtype=dtype, pin_memory=True) for _ in range(2)]
    for h in host_in:
        h.copy_(x.view(-1).cpu())
    host_out = [torch.empty(n, dtype=dtype, pin_memory=True) for _ in range(2)]
    return host_in, host_out


def _find_reference():
    cands = []
    env = os.environ.get("LZ_REFERENCE_DIR")
    if env:
        cands += [env, os.path.join(env, REF_SUBDIR)]
    cands += [os.path.join(ROOT, "baseline", "_ref", REF_SUBDIR), os.path.join(ROOT, "baseline", "_ref")]
    for d in cands:
        if os.path.isfile(os.path.join(d, "benchmark_both.py")):
            return d, cands
    return None, cands


def reference_arm(args) -> int:
    """The reference's own NCCL benchmark functions, imported unchanged."""
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    rank_env = int(os.environ.get("RANK", "0"))
    d, checked = _find_reference()
    if d is None:
        if rank_env == 0:
            print(json.dumps({"impl": "reference", "metric": METRIC, "n_gpus": world_env,
                              "unavailable": "reference scripts not found; checked: " + ", ".join(checked)}))
        return 0
    import torch
    import torch.distributed as dist

    sys.path.insert(0, d)
    import benchmark_both as ref_both  # noqa: E402  (reference module, unmodified)
    import nccl_standard_allreduce as ref_std  # noqa: E402

    rank, world, local, ctrl = _setup(args)
    nbytes = args.size_mb << 20
    n = nbytes // 2  # the reference's main(): num_elements = size_bytes // 2 (bf16)
    bus = 2.0 * (world - 1) / world if world > 1 else 1.0
    Sampler = _clock_sampler_cls()

    torch.cuda.synchronize()
    dist.barrier(group=ctrl)
    sampler = Sampler([local]).start()
    cuda_ms, wall_ms = ref_both.bench_standard(n, num_warmup=args.warmup, num_iters=args.steps)
    torch.cuda.synchronize()
    dist.barrier(group=ctrl)
    sampler.stop()
    ms = _max_over_ranks(cuda_ms, ctrl)
    wall = _max_over_ranks(wall_ms, ctrl)
    algbw = nbytes / (ms * 1e-3) / 1e9
    torch.cuda.empty_cache()

    dist.barrier(group=ctrl)
    std_ms, _, _ = ref_std.benchmark_allreduce(nbytes, world, num_warmup=args.warmup, num_iters=args.steps)
    std_ms = _max_over_ranks(std_ms, ctrl)
    std_alg = nbytes / (std_ms * 1e-3) / 1e9
    torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e:
        # the reference's public API for the collective is torch.distributed.all_reduce
        dtype = ref_both.DTYPE
        x = ref_both.make_rand_tensor(n)
        host_in, host_out = _pinned_inputs(x, n, dtype)
        dev_in = [x, torch.empty_like(x)]

        def step(buf, _out):
            dist.all_reduce(buf, op=dist.ReduceOp.SUM)

        e_ms, _ = _e2e(step, host_in, host_out, dev_in, dev_in, args.steps, args.warmup, ctrl, local)
        e_alg = nbytes / (e_ms * 1e-3) / 1e9
        e2e = {"value": round(world * e_alg * bus, 3), "unit": "GB/s", "ms_per_step": round(e_ms, 4),
               "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
               "api": "torch.distributed.all_reduce (the reference's collective call)"}
    if rank == 0:
        print(json.dumps({
            "impl": "reference",
            "metric": METRIC,
            "value": round(world * algbw * bus, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: uniform[-1, 1] (the reference's make_rand_tensor/reset_rand)",
            "config": {
                "model": f"allreduce sum bfloat16 {args.size_mb} MiB per rank",
                "global_batch": world, "seq_len": n, "parallelism": f"dp{world}",
                "code": f"{REF_SUBDIR}/benchmark_both.py bench_standard (unmodified, from {d})",
                "timed_loop": "reference's own: reset_rand refill + dist.all_reduce per iteration",
                "busbw_GBps_per_rank": round(algbw * bus, 3), "algbw_GBps": round(algbw, 3),
                "wall_ms_per_step": round(wall, 4),
                "nccl_standard_fp32_no_fill": {"code": f"{REF_SUBDIR}/nccl_standard_allreduce.py benchmark_allreduce",
                                               "ms": round(std_ms, 4),
                                               "busbw_GBps_per_rank": round(std_alg * bus, 3)},
                "l2": "1 GiB inputs per rank exceed the 126 MB L2; no flush between steps",
                "timing": "CUDA events inside the reference function, max over ranks",
            },
            "clocks": sampler.summary(),
            "e2e": e2e,
            "gpu_launches": 0,
        }), flush=True)
    dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)

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

        e2e_bytes = 0 if args.no_e2e else 2 * nbytes
        cfg = Config(user_bytes=2 * nbytes + e2e_bytes + 64 * MiB, stage_bytes=64 * MiB, oneshot_bytes=8 * MiB)
        comm = lz.init(config=cfg)
        x = comm.empty(n, dtype)
        y = comm.empty(n, dtype)
        x.copy_(_input(rank, n, dtype))
        algo = args.algo
        if algo == "auto":
            algo = lz.select_algo(nbytes, world, comm.has_multicast, True, comm.config)

        def step():
            comm.allreduce_(x, y, algo=algo)

        launches_per_step = 1
    else:
        algo = "nccl"
        x = _input(rank, n, dtype)
        y = x

        def step():
            dist.all_reduce(x)

    ms, clocks = _timed(step, args.steps, args.warmup, ctrl, [local])
    if comm is not None:
        comm.check()
    algbw, busbw = bw(ms)

    nccl_cmp = None
    z1 = None
    if args.impl == "ours" and world > 1 and not args.no_nccl_compare:
        z = x.clone()
        n_ms, _ = _timed(lambda: dist.all_reduce(z), args.steps, args.warmup, ctrl, [local])
        z.copy_(x)
        dist.all_reduce(z)  # one all_reduce of the same inputs, for the accuracy comparison
        z1 = z
        torch.cuda.synchronize()
        nccl_cmp = {"ms": round(n_ms, 4), "busbw_GBps_per_rank": round(bw(n_ms)[1], 3),
                    "ours_over_nccl": round(n_ms / ms, 4)}

    check = None
    if args.impl == "ours" and not args.no_check:
        ys = {"ours": y}
        if z1 is not None:
            ys["nccl_all_reduce"] = z1
        check = _check_full(ys, world, n, dtype, ctrl)
    z1 = None
    torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e:
        host_in, host_out = _pinned_inputs(x, n, dtype)
        if args.impl == "ours":
            import results_b200 as lz

            dev_in = [comm.empty(n, dtype), x]
            dev_out = [comm.empty(n, dtype), y]

            def e2e_fn(buf, out):
                lz.allreduce(buf, algo="auto", out=out, comm=comm)
        else:
            dev_in = [x, torch.empty_like(x)]
            dev_out = dev_in

            def e2e_fn(buf, _out):
                dist.all_reduce(buf)

        e_ms, _ = _e2e(e2e_fn, host_in, host_out, dev_in, dev_out, args.steps, args.warmup, ctrl, local)
        _, e_bus = bw(e_ms)
        e2e = {"value": round(world * e_bus, 3), "unit": "GB/s", "ms_per_step": round(e_ms, 4),
               "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
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
                "n1_note": "world 1: the allreduce is the identity; out-of-place it is one local copy",
                "baseline_ref": ("reference LZip two-shot at 1 GB as a whole-job aggregate: ws=2 109.36 GB/s, "
                                 "ws=8 428.8 GB/s (53.60 busbw per rank); H200 + EFA; none published for 1 or 4"),
            },
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
        }
        if comm is not None:
            out["config"]["multicast"] = comm.has_multicast
        if nccl_cmp is not None:
            out["config"]["nccl_same_harness"] = nccl_cmp
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
