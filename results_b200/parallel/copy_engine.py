"""Allreduce paths that move data without SM copy loops.

* :func:`ce_allreduce` -- two-shot whose bytes cross NVLink by copy-engine
  DMA (cudaMemcpyAsync into / from peer-mapped heap memory) while the SMs only
  accumulate (csrc/lz_copy_engine.cu). Symmetric, distinct input and output
  take the zero-copy pipelined path (reduce-scatter pushes, per-chunk reduce,
  all-gather pushes on two side streams, ``pipes`` chunks per slice, 0 =
  automatic); other buffers go through the communicator stage.
* :func:`hoststaged_allreduce` -- PCIe emulation: every exchange goes
  through pinned, cross-process shared host memory (D2H, host barrier, H2D),
  the B200 counterpart of the reference's host-staged mode and of its
  "peer access disabled" (``p2p_nopa``) baseline
  (single_node_nccl_allreduce_benchmark/memcpy_p2p_allreduce_kernel.cu:233-309,
  single_node_nccl_allreduce_benchmark/benchmark_both.py:182-213).
"""
from __future__ import annotations

from multiprocessing import shared_memory

import torch
import torch.distributed as dist

from ..utils.dtypes import lz_dtype


def ce_allreduce(t: torch.Tensor, out: torch.Tensor | None = None, comm=None, pipes: int = 0) -> torch.Tensor:
    """Copy-engine two-shot sum-allreduce (in place unless ``out`` is given)."""
    from .allreduce import get_comm, init

    comm = comm or get_comm() or init()
    return comm.allreduce_(t, out, algo="ce", pipes=pipes)


def is_zero_copy(comm, t: torch.Tensor, out: torch.Tensor | None = None) -> bool:
    """True when (t, out) take the zero-copy pipelined copy-engine path."""
    out = t if out is None else out
    return bool(comm._lib.lz_ce_allreduce_is_zero_copy(comm.handle, t.data_ptr(), out.data_ptr(), t.numel(),
                                                        lz_dtype(t.dtype)))


class _HostStage:
    """Per-rank pinned shared-memory segment, opened by every peer."""

    def __init__(self, group, nbytes: int, tag: str):
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nbytes = nbytes
        self.mine = shared_memory.SharedMemory(name=f"lzhs_{tag}_{self.rank}", create=True, size=nbytes)
        dist.barrier(group=group)
        self.seg = {}
        for r in range(self.world):
            self.seg[r] = self.mine if r == self.rank else shared_memory.SharedMemory(name=f"lzhs_{tag}_{r}")
        self.views = {}
        cudart = torch.cuda.cudart()
        for r, m in self.seg.items():
            t = torch.frombuffer(m.buf, dtype=torch.uint8)
            cudart.cudaHostRegister(t.data_ptr(), nbytes, 0)
            self.views[r] = t

    def close(self):
        cudart = torch.cuda.cudart()
        for t in self.views.values():
            cudart.cudaHostUnregister(t.data_ptr())
        self.views.clear()
        for r, m in self.seg.items():
            m.close()
        self.mine.unlink()


_HS: dict = {}


def hoststaged_allreduce(t: torch.Tensor, group=None, ctrl=None) -> torch.Tensor:
    """Two-shot through shared pinned host memory (no GPU peer access)."""
    ws = dist.get_world_size(group)
    if ws == 1:
        return t
    rank = dist.get_rank(group)
    ctrl = ctrl or group
    nbytes = t.numel() * t.element_size()
    key = (id(group), nbytes)
    if key not in _HS:
        tag = [f"{torch.randint(0, 1 << 30, (1,)).item():x}" if rank == 0 else None]
        dist.broadcast_object_list(tag, src=0, group=ctrl)
        _HS[key] = _HostStage(ctrl, 2 * nbytes, tag[0])
    hs = _HS[key]
    n = t.numel()
    c = n // ws
    es = t.element_size()
    flat = t.view(-1)
    mine_host = hs.views[rank][:nbytes].view(t.dtype)
    mine_host.copy_(flat, non_blocking=True)  # D2H of every slice peers need
    torch.cuda.current_stream().synchronize()
    dist.barrier(group=ctrl)
    lo, hi = rank * c, (n if rank == ws - 1 else (rank + 1) * c)
    acc = None
    for r in range(ws):  # rank order, fp32
        src = flat[lo:hi] if r == rank else hs.views[r][:nbytes].view(t.dtype)[lo:hi].to(t.device, non_blocking=True)
        acc = src.float().clone() if acc is None else acc + src.float()
    flat[lo:hi].copy_(acc)
    res_host = hs.views[rank][nbytes:2 * nbytes].view(t.dtype)
    res_host[lo:hi].copy_(flat[lo:hi], non_blocking=True)
    torch.cuda.current_stream().synchronize()
    dist.barrier(group=ctrl)
    for r in range(ws):
        if r != rank:
            plo, phi = r * c, (n if r == ws - 1 else (r + 1) * c)
            flat[plo:phi].copy_(hs.views[r][nbytes:2 * nbytes].view(t.dtype)[plo:phi], non_blocking=True)
    torch.cuda.current_stream().synchronize()
    dist.barrier(group=ctrl)
    return t


def close_host_stages():
    for hs in _HS.values():
        hs.close()
    _HS.clear()
