"""Topology and link probes: device properties, peer access and NVLink
performance rank, NVLS multicast support, and a P2P copy-bandwidth probe.

Reference counterparts: single_node_nccl_allreduce_benchmark/p2p_bw_test.cu:4-26 and
single_node_nccl_allreduce_benchmark/test_p2p_bandwidth.py:20-83 (GPU0 -> GPU1
copy with peer access on and off).
"""
from __future__ import annotations

import ctypes as C
import time

import torch

from .. import _native


def device_info(device: int) -> dict:
    L = _native.cuda()
    sms, mc, ma, mi = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    mem = C.c_size_t()
    _native.check(L.lz_device_info(device, C.byref(sms), C.byref(mc), C.byref(ma), C.byref(mi), C.byref(mem)),
                  "device info")
    return {"device": device, "sm_count": sms.value, "multicast": bool(mc.value),
            "cc": f"{ma.value}.{mi.value}", "total_mem": mem.value}


def peer_matrix() -> dict:
    """{(i, j): {"access": bool, "perf_rank": int, "native_atomics": bool}} for all GPU pairs."""
    L = _native.cuda()
    n = torch.cuda.device_count()
    out = {}
    for i in range(n):
        for j in range(n):
            if i == j:
                continue
            can, pr, na = C.c_int(), C.c_int(), C.c_int()
            _native.check(L.lz_can_access_peer(i, j, C.byref(can)), "peer access")
            _native.check(L.lz_nvlink_p2p_attr(i, j, C.byref(pr), C.byref(na)), "p2p attr")
            out[(i, j)] = {"access": bool(can.value), "perf_rank": pr.value, "native_atomics": bool(na.value)}
    return out


def p2p_copy_bandwidth(src: int = 0, dst: int = 1, nbytes: int = 1 << 30, iters: int = 10,
                       via_host: bool = False) -> float:
    """GB/s of a src->dst copy (device timing on the destination stream).

    ``via_host=True`` stages through pinned host memory: the path taken when
    peer access is unavailable (the reference's "peer access disabled" case).
    """
    a = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{src}")
    b = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dst}")
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) if via_host else None
    with torch.cuda.device(dst):
        def once():
            if via_host:
                h.copy_(a, non_blocking=False)
                b.copy_(h, non_blocking=True)
            else:
                b.copy_(a, non_blocking=True)
        once()
        torch.cuda.synchronize(src)
        torch.cuda.synchronize(dst)
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            once()
        e1.record()
        torch.cuda.synchronize(dst)
        ms = e0.elapsed_time(e1) / iters
        if via_host:  # the D2H half is synchronous on the host; use wall time
            ms = (time.perf_counter() - t0) * 1e3 / iters
    return nbytes / (ms * 1e-3) / 1e9


def summary() -> dict:
    n = torch.cuda.device_count()
    return {"devices": [device_info(i) for i in range(n)],
            "peers": {f"{i}->{j}": v for (i, j), v in peer_matrix().items()} if n > 1 else {}}
