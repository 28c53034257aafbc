"""Helpers to run a function on W child processes (one per GPU or gloo CPU rank).

Each child initialises torch.distributed on 127.0.0.1 with a short timeout so
that ranks waiting on a dead peer end with an error instead of hanging.
"""
from __future__ import annotations

import datetime
import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _child(rank, world, port, backend, fn, args, q, env):
    try:
        os.environ.update(env)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["RANK"] = str(rank)
        os.environ["WORLD_SIZE"] = str(world)
        os.environ["LOCAL_RANK"] = str(rank)
        os.environ["LOCAL_WORLD_SIZE"] = str(world)
        import torch
        import torch.distributed as dist

        if backend == "nccl":
            torch.cuda.set_device(rank)
        kw = dict(backend=backend, rank=rank, world_size=world,
                  timeout=datetime.timedelta(seconds=float(env.get("LZ_TEST_PG_TIMEOUT", "120"))))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", rank)
        dist.init_process_group(**kw)
        res = fn(rank, world, *args)
        q.put((rank, "ok", res))
        if env.get("LZ_TEST_NO_FINAL_BARRIER") != "1":
            try:
                dist.barrier()
            except Exception:
                pass
        try:
            dist.destroy_process_group()
        except Exception:
            pass
    except BaseException:
        q.put((rank, "error", traceback.format_exc()))


def run_ranks(fn, world: int, backend: str = "gloo", args=(), timeout: float = 600.0, env=None,
              allow_missing: bool = False):
    """Run fn(rank, world, *args) on `world` processes; returns per-rank results.

    Raises AssertionError carrying the first child traceback on failure.
    """
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    env = dict(env or {})
    procs = [ctx.Process(target=_child, args=(r, world, port, backend, fn, args, q, env), daemon=False)
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    errors = []
    import queue as _queue
    import time

    deadline = time.time() + timeout
    while len(results) + len(errors) < world and time.time() < deadline:
        try:
            rank, status, payload = q.get(timeout=1.0)
        except _queue.Empty:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
            continue
        if status == "ok":
            results[rank] = payload
        else:
            errors.append((rank, payload))
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    if errors:
        rank, tb = errors[0]
        raise AssertionError(f"rank {rank} failed:\n{tb}")
    if len(results) < world and not allow_missing:
        raise AssertionError(f"only {len(results)}/{world} ranks reported (timeout or crash)")
    return [results.get(r) for r in range(world)]
