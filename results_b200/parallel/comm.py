"""Communicator: bootstrap of the symmetric heap and device-side state.

One process per GPU. The control plane (rendezvous, barriers, fd exchange
ordering) runs over a gloo process group; the data plane is NVLink peer
memory mapped through cuMem VMM plus an optional NVLS multicast object.

Reference counterpart: the per-driver ``setup()`` + IPC-handle all_gather of
single_node_nccl_allreduce_benchmark/p2p_twoshot_allreduce.py:32-62 and the MPI
bootstrap of back_up/mpi_hello.cpp:61-122.
"""
from __future__ import annotations

import atexit
import ctypes as C
import os
import secrets
import weakref

import torch
import torch.distributed as dist

from .. import _native
from ..config import Config
from ..utils.dtypes import lz_dtype

ALGOS = {
    "oneshot": 0,
    "twoshot": 1,
    "nvls": 2,
    "ring": 3,
    "rhd": 4,
    "nvls_oneshot": 5,
    "ll": 6,
}


class _CudaBuf:
    """Minimal __cuda_array_interface__ view of raw device memory."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {
            "shape": (nbytes,),
            "typestr": "|u1",
            "data": (ptr, False),
            "version": 3,
            "strides": None,
            "stream": None,
        }


_LIVE: "weakref.WeakSet[Communicator]" = weakref.WeakSet()


def _control_group(group):
    """A gloo group over the same ranks for host-side barriers."""
    if group is None and dist.get_backend() == "gloo":
        return None
    if group is not None and dist.get_backend(group) == "gloo":
        return group
    ranks = dist.get_process_group_ranks(group) if group is not None else list(
        range(dist.get_world_size()))
    return dist.new_group(ranks=ranks, backend="gloo")


class Communicator:
    """Symmetric heap + device communicator for one process group.

    Creation is collective over ``group``. All collectives of one
    communicator must be issued on one stream at a time (stream order is what
    keeps the per-call epoch consistent across ranks).
    """

    def __init__(self, group=None, config: Config | None = None, device: int | None = None):
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialized first")
        self.config = config or Config.from_env()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.cuda.current_device() if device is None else device
        self.ctrl = _control_group(group)
        self._lib = _native.cuda()
        self._heap = C.c_void_p()
        self._comm = C.c_void_p()
        self._closed = False
        tag = [secrets.token_hex(6) if self.rank == 0 else None]
        dist.broadcast_object_list(tag, src=self._global(0), group=self.ctrl)
        self.tag = f"{os.getpid() if self.world == 1 else tag[0]}"
        L = self._lib
        cfg = self.config
        with torch.cuda.device(self.device):
            _native.check(L.lz_heap_create(self.device, self.rank, self.world, cfg.total_heap_bytes(),
                                           int(cfg.use_multicast), self.tag.encode(),
                                           C.byref(self._heap)), "lz_heap_create")
            _native.check(L.lz_heap_serve(self._heap), "lz_heap_serve")
            self.barrier_host()
            _native.check(L.lz_heap_connect(self._heap), "lz_heap_connect")
            self.barrier_host()
            # NVLS multicast: create -> attach (add device) -> bind -> map
            _native.check(L.lz_mc_create(self._heap), "lz_mc_create")
            self.barrier_host()
            _native.check(L.lz_mc_attach(self._heap), "lz_mc_attach")
            self.barrier_host()
            _native.check(L.lz_mc_bind(self._heap), "lz_mc_bind")
            self.barrier_host()
            _native.check(L.lz_mc_map(self._heap), "lz_mc_map")
            self.barrier_host()
            L.lz_heap_stop_serving(self._heap)
            _native.check(L.lz_comm_create(self._heap, cfg.oneshot_bytes, cfg.stage_bytes,
                                           cfg.timeout_s, C.byref(self._comm)), "lz_comm_create")
            self.barrier_host()
        self.heap_bytes = L.lz_heap_size(self._heap)
        self.has_multicast = bool(L.lz_heap_has_mc(self._heap))
        self._user_off = L.lz_comm_user_offset(self._comm)
        self._bump = self._user_off
        self._local_base = L.lz_heap_ptr(self._heap, self.rank)
        props = torch.cuda.get_device_properties(self.device)
        self.sm_count = props.multi_processor_count
        _LIVE.add(self)

    # ------------------------------------------------------------------ utils
    def _global(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def barrier_host(self) -> None:
        dist.barrier(group=self.ctrl)

    @property
    def handle(self):
        return self._comm

    def peer_ptr(self, rank: int, offset: int = 0) -> int:
        return self._lib.lz_heap_ptr(self._heap, rank) + offset

    def multicast_ptr(self, offset: int = 0) -> int | None:
        p = self._lib.lz_heap_mc_ptr(self._heap)
        return None if not p else p + offset

    # -------------------------------------------------------- symmetric memory
    def alloc(self, nbytes: int, align: int = 256) -> int:
        """Collective bump allocation in the user region; returns the heap offset.

        Every rank must make the same sequence of calls so that offsets match.
        """
        off = (self._bump + align - 1) // align * align
        if off + nbytes > self.heap_bytes:
            raise MemoryError(f"symmetric heap exhausted: need {nbytes} bytes at {off}, "
                              f"heap is {self.heap_bytes} bytes (raise Config.user_bytes)")
        self._bump = off + nbytes
        return off

    def reset_alloc(self) -> None:
        self._bump = self._user_off

    def tensor_at(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """Tensor view of this rank's own heap memory at ``offset``.

        There is deliberately no way to get a torch view of a peer's heap:
        only this library's kernels and copy-engine transfers touch peer
        memory, never a PyTorch or other library kernel.
        """
        shape = tuple(shape) if isinstance(shape, (tuple, list, torch.Size)) else (int(shape),)
        numel = 1
        for s in shape:
            numel *= int(s)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        if offset < self._user_off or offset + nbytes > self.heap_bytes:
            raise ValueError(f"heap range [{offset}, {offset + nbytes}) is outside the user region "
                             f"[{self._user_off}, {self.heap_bytes})")
        buf = _CudaBuf(self._local_base + offset, max(nbytes, 1), self)
        t = torch.as_tensor(buf, device=f"cuda:{self.device}")[:nbytes]
        return t.view(dtype).view(shape)

    def empty(self, shape, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """Allocate a symmetric tensor (collective): zero-copy for every collective."""
        shape = tuple(shape) if isinstance(shape, (tuple, list, torch.Size)) else (int(shape),)
        numel = 1
        for s in shape:
            numel *= int(s)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        off = self.alloc(nbytes)
        return self.tensor_at(off, shape, dtype)

    def is_symmetric(self, t: torch.Tensor) -> bool:
        p = t.data_ptr()
        return self._local_base + self._user_off <= p < self._local_base + self.heap_bytes

    # ------------------------------------------------------------ collectives
    def allreduce_(self, inp: torch.Tensor, out: torch.Tensor | None = None, algo: str = "twoshot",
                   nblocks: int = 0, nthreads: int = 0, stream=None, pipes: int = 0) -> torch.Tensor:
        """Native sum-allreduce of a contiguous CUDA tensor (in place by default).

        ``algo="ce"`` is the copy-engine two-shot (``pipes`` chunks per slice,
        0 = automatic); every other algorithm is one kernel launch.
        """
        if out is None:
            out = inp
        if not (inp.is_contiguous() and out.is_contiguous()):
            raise ValueError("allreduce needs contiguous tensors")
        if inp.numel() != out.numel() or inp.dtype != out.dtype:
            raise ValueError("input and output must match in numel and dtype")
        for t in (inp, out):
            if not t.is_cuda or t.device.index != self.device:
                raise ValueError(f"allreduce tensors must be on cuda:{self.device} (got {t.device})")
        s = stream or torch.cuda.current_stream(self.device)
        if algo == "ce":
            rc = self._lib.lz_ce_allreduce(self._comm, inp.data_ptr(), out.data_ptr(), inp.numel(),
                                           lz_dtype(inp.dtype), int(pipes), s.cuda_stream)
            _native.check(rc, "allreduce[ce]")
            return out
        nb = nblocks or self.config.sm_budget
        nt = nthreads or self.config.nthreads
        rc = self._lib.lz_allreduce(self._comm, inp.data_ptr(), out.data_ptr(), inp.numel(),
                                    lz_dtype(inp.dtype), ALGOS[algo], nb, nt, s.cuda_stream)
        _native.check(rc, f"allreduce[{algo}]")
        return out

    def device_barrier(self, stream=None) -> None:
        s = stream or torch.cuda.current_stream(self.device)
        _native.check(self._lib.lz_barrier(self._comm, s.cuda_stream), "barrier")

    # ------------------------------------------------------------ health
    def status(self) -> int:
        return self._lib.lz_comm_status(self._comm)

    def check(self) -> None:
        """Raise CollectiveTimeout if any device wait gave up (call after a sync)."""
        st = self.status()
        if st:
            code, phase, peer, block = st & 0xFF, (st >> 8) & 0xFF, (st >> 16) & 0xFF, (st >> 24) & 0xFF
            raise _native.CollectiveTimeout(
                f"rank {self.rank}: device wait failed (code {code}) in phase {phase} "
                f"waiting for rank {peer} (block {block}); communicator must be recreated")

    def test_wait_timeout(self, timeout_s: float = 0.2) -> None:
        """Launch a kernel whose bounded wait must expire (failure-path test hook)."""
        s = torch.cuda.current_stream(self.device)
        _native.check(self._lib.lz_test_wait_timeout(self._comm, C.c_double(timeout_s), s.cuda_stream),
                      "test wait")

    def clear_status(self) -> None:
        self._lib.lz_comm_clear_status(self._comm)

    def attach_heartbeat(self, period_s: float = 0.2):
        """Start publishing liveness in the store; `guard()` then checks peers."""
        from ..utils.health import Heartbeat

        self._hb = Heartbeat(self.rank, self.world, period_s=period_s)
        return self._hb

    def guard(self, max_age_s: float = 2.0) -> None:
        """Raise PeerLost before launching if a peer left or stopped heart-beating."""
        hb = getattr(self, "_hb", None)
        if hb is not None:
            hb.check(max_age_s)

    def epoch(self) -> int:
        v = C.c_uint64()
        s = torch.cuda.current_stream(self.device)
        _native.check(self._lib.lz_comm_epoch(self._comm, C.byref(v), s.cuda_stream), "epoch")
        return v.value

    # ------------------------------------------------------------ teardown
    def abandon(self) -> None:
        """Local, non-collective teardown for failure paths (no peer barrier).

        Only call when none of this rank's kernels are in flight. Peers keep
        their own imports of this rank's memory alive until they tear down.
        """
        if self._closed:
            return
        self._closed = True
        import sys

        w = sys.modules.get("results_b200.parallel.weights")
        if w is not None:  # cached weight engines hold this communicator
            w._ENGINES.pop(self, None)
        try:
            torch.cuda.synchronize(self.device)
        except Exception:
            pass
        hb = getattr(self, "_hb", None)
        if hb is not None:
            hb.stop()
        self._lib.lz_comm_destroy(self._comm)
        self._lib.lz_heap_destroy(self._heap)

    def close(self) -> None:
        """Collective teardown: barrier, then unmap peers and unbind multicast."""
        if self._closed:
            return
        self._closed = True
        import sys

        w = sys.modules.get("results_b200.parallel.weights")
        if w is not None:  # cached weight engines hold this communicator
            w._ENGINES.pop(self, None)
        try:
            torch.cuda.synchronize(self.device)
            self.barrier_host()
        except Exception:
            pass
        L = self._lib
        L.lz_comm_destroy(self._comm)
        try:
            self.barrier_host()
        except Exception:
            pass
        L.lz_heap_destroy(self._heap)

    def __del__(self):
        pass


def _close_all():
    for c in list(_LIVE):
        try:
            c.close()
        except Exception:
            pass


atexit.register(_close_all)
