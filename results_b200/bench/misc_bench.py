"""Small benches of the reference's auxiliary tools.

    python -m results_b200.bench.misc_bench p2p        # GPU0 -> GPU1 copy, peer vs host-staged
    python -m results_b200.bench.misc_bench fp8        # fp8 pair pack/unpack GB/s + round trip
    torchrun --nproc-per-node 2 -m results_b200.bench.misc_bench memcpy   # copy-engine vs host-staged two-shot

Counterparts: single_node_nccl_allreduce_benchmark/test_p2p_bandwidth.py:20-83,
back_up/fp8_e4m3fn_pack_benchmark.cu:192-299 (256 MiB random bytes, self-checking
round trip), single_node_nccl_allreduce_benchmark/bench_memcpy_p2p.py:37-98 (pipes
{1,2,4,8,16}, pieces below 512 KB skipped, best reported).
"""
from __future__ import annotations

import datetime
import os
import sys

import torch


def bench_p2p():
    from results_b200.utils import topology

    n = torch.cuda.device_count()
    if n < 2:
        print("needs 2 GPUs")
        return
    for size in (1 << 20, 64 << 20, 1 << 30):
        peer = topology.p2p_copy_bandwidth(0, 1, size)
        host = topology.p2p_copy_bandwidth(0, 1, size, via_host=True)
        print(f"{size >> 20:5d} MB  peer {peer:8.1f} GB/s   host-staged {host:8.1f} GB/s", flush=True)


def bench_fp8(mib: int = 256, iters: int = 20):
    from results_b200.ops import fp8

    g = torch.Generator().manual_seed(12345)
    x = torch.randint(0, 256, (mib << 20,), dtype=torch.uint8, generator=g).cuda()
    for kind in ("e4m3", "e5m2"):
        w = fp8.pack_fp8(x, kind)
        y = fp8.unpack_fp8(w, kind)
        ok = torch.equal(x, y)
        for name, fn in (("pack", lambda: fp8.pack_fp8(x, kind)), ("unpack", lambda: fp8.unpack_fp8(w, kind))):
            for _ in range(3):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / iters
            gbs = 2 * x.numel() / (ms * 1e-3) / 1e9  # bytes read + written
            print(f"{kind} {name:6s}: {ms:.3f} ms  {gbs:.1f} GB/s (read+write)  roundtrip_ok={ok}", flush=True)


def bench_memcpy():
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    ctrl = dist.new_group(backend="gloo")
    import results_b200 as lz
    from results_b200.config import Config, MiB
    from results_b200.parallel import copy_engine

    world = dist.get_world_size()
    comm = lz.init(config=Config(user_bytes=16 * MiB, stage_bytes=2560 * MiB))
    for size in (4 << 20, 64 << 20, 256 << 20, 1 << 30):
        x = torch.randn(size // 2, device="cuda").to(torch.bfloat16)
        best = None
        for pipes in (1, 2, 4, 8, 16):
            if size // world // pipes < (512 << 10):
                continue
            for _ in range(2):
                copy_engine.ce_allreduce(x, comm=comm, pipes=pipes)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                copy_engine.ce_allreduce(x, comm=comm, pipes=pipes)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 5
            t = torch.tensor([ms], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctrl)
            ms = t.item()
            if best is None or ms < best[0]:
                best = (ms, pipes)
        import time

        t0 = time.perf_counter()
        copy_engine.hoststaged_allreduce(x, ctrl=ctrl)
        torch.cuda.synchronize()
        host_ms = (time.perf_counter() - t0) * 1e3
        if rank == 0:
            bus = 2 * (world - 1) / world
            print(f"{size >> 20:5d} MB  copy-engine best {best[0]:.3f} ms (pipes={best[1]}, busbw "
                  f"{size / best[0] / 1e6 * bus:.1f} GB/s)  host-staged {host_ms:.1f} ms", flush=True)
    copy_engine.close_host_stages()
    lz.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "fp8"
    {"p2p": bench_p2p, "fp8": bench_fp8, "memcpy": bench_memcpy}[what]()
