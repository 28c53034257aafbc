"""Single-GPU emulation of R ranks for testing the multi-rank kernels.

The R "ranks" each own a heap allocated on the same GPU; a collective runs as
ONE cooperative launch of grid (G, R) so that every block that waits on
another is guaranteed to be co-resident. This exercises the exact kernel
bodies (barriers, flags, partitioning, reduction order) used across GPUs,
without NVLink and without NVLS (no multicast object with one device).
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _native
from ..utils.dtypes import lz_dtype
from .comm import ALGOS, _CudaBuf

MiB = 1 << 20


class EmulatedWorld:
    def __init__(self, world: int, heap_bytes: int = 256 * MiB, oneshot_bytes: int = 4 * MiB,
                 stage_bytes: int = 64 * MiB, timeout_s: float = 5.0):
        self.world = world
        self._lib = _native.cuda()
        self._emu = C.c_void_p()
        _native.check(self._lib.lz_emu_create(world, heap_bytes, oneshot_bytes, stage_bytes,
                                              timeout_s, C.byref(self._emu)), "lz_emu_create")
        self.heap_bytes = heap_bytes
        self._user_off = self._lib.lz_emu_user_offset(self._emu)
        self._bump = self._user_off
        self.device = torch.cuda.current_device()

    def empty(self, shape, dtype) -> list[torch.Tensor]:
        """Symmetric allocation: one tensor per emulated rank at the same offset."""
        shape = tuple(shape) if isinstance(shape, (tuple, list)) else (int(shape),)
        numel = 1
        for s in shape:
            numel *= s
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        off = (self._bump + 255) // 256 * 256
        if off + nbytes > self.heap_bytes:
            raise MemoryError("emulated heap exhausted")
        self._bump = off + nbytes
        out = []
        for r in range(self.world):
            base = self._lib.lz_emu_heap_ptr(self._emu, r)
            buf = _CudaBuf(base + off, max(nbytes, 1), self)
            t = torch.as_tensor(buf, device=f"cuda:{self.device}")[:nbytes]
            out.append(t.view(dtype).view(shape))
        return out

    def allreduce(self, ins, outs, algo: str = "twoshot", nblocks: int = 0, nthreads: int = 0):
        R = self.world
        assert len(ins) == len(outs) == R
        arr_in = (C.c_void_p * R)(*[t.data_ptr() for t in ins])
        arr_out = (C.c_void_p * R)(*[t.data_ptr() for t in outs])
        s = torch.cuda.current_stream()
        rc = self._lib.lz_emu_allreduce(self._emu, arr_in, arr_out, ins[0].numel(),
                                        lz_dtype(ins[0].dtype), ALGOS[algo], nblocks, nthreads,
                                        s.cuda_stream)
        _native.check(rc, f"emulated allreduce[{algo}]")

    def compressed_allreduce(self, ins, outs, nblocks: int = 0, hybrid: bool = False, level="ans",
                             chunk_elems: int = 0, stage_local: bool = False, trace=None):
        """trace: int64 CUDA tensor [R, nblocks, phases] for the kernel's phase tracer."""
        from . import compressed  # noqa: F401  (declares the native signature)
        from ..ops import codec

        R = self.world
        arr_in = (C.c_void_p * R)(*[t.data_ptr() for t in ins])
        arr_out = (C.c_void_p * R)(*[t.data_ptr() for t in outs])
        rc = self._lib.lz_emu_compressed_allreduce_traced(self._emu, arr_in, arr_out, ins[0].numel(),
                                                   lz_dtype(ins[0].dtype), nblocks,
                                                   (2 if hybrid else 0) | 4 * codec.level_code(level) |
                                                   (8 if stage_local else 0), chunk_elems,
                                                   trace.data_ptr() if trace is not None else None,
                                                   torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "emulated compressed allreduce")

    def weight_transfer(self, src: int, dsts, tensors, encode: bool = True, nblocks: int = 16,
                        kslots: int = 3, broadcast_all: bool = False):
        """One transfer from emulated rank `src` to `dsts`; tensors[r] is rank r's list."""
        from . import weights

        R = self.world
        if not hasattr(self, "_wx_seq"):
            self._wx_seq = {}
        mask = 0
        for d in dsts:
            mask |= 1 << d
        seqs = [0] * (8 * R)
        for d in dsts:
            key = ("b", src) if broadcast_all else (src, d)
            k = self._wx_seq.get(key, 0) + (0 if broadcast_all and d != dsts[0] else 1)
            self._wx_seq[key] = k
        for r in range(R):
            for q in range(8):
                if broadcast_all:
                    seqs[8 * r + q] = self._wx_seq[("b", src)]
                elif r == src:
                    seqs[8 * r + q] = self._wx_seq.get((src, q), 0) if q in dsts else 0
                elif r in dsts:
                    seqs[8 * r + q] = self._wx_seq[(src, r)]
        keep = []
        ptrs = []
        ntg = None
        for r in range(R):
            ts = tensors[r] if tensors[r] is not None else tensors[src]
            d, n = weights.build_descriptors(ts, [encode] * len(ts), f"cuda:{self.device}")
            keep.append(d)
            ptrs.append(d.data_ptr())
            ntg = n
        arr = (C.c_void_p * R)(*ptrs)
        sq = (C.c_uint64 * (8 * R))(*seqs)
        flags = int(broadcast_all) | (2 if encode == 2 else 0)  # bit 1: PACK-level records
        rc = self._lib.lz_emu_weight_transfer(self._emu, src, mask, arr, ntg, nblocks, kslots,
                                              flags, sq, torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "emulated weight transfer")

    def all_to_all(self, ins, outs, compress: bool = False, nblocks: int = 0):
        """ins[r] / outs[r]: rank r's W equal chunks (outs symmetric or not)."""
        from . import alltoall  # noqa: F401  (declares the native signature)

        R = self.world
        x = ins[0]
        dt = lz_dtype(x.dtype) if x.dtype in alltoall.COMPRESSIBLE else 3
        chunk = x.numel() // R * (1 if dt != 3 else x.element_size())
        arr_in = (C.c_void_p * R)(*[t.data_ptr() for t in ins])
        arr_out = (C.c_void_p * R)(*[t.data_ptr() for t in outs])
        from .alltoall import enc_code

        rc = self._lib.lz_emu_all_to_all(self._emu, arr_in, arr_out, chunk, dt, enc_code(compress), nblocks,
                                         torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "emulated all_to_all")

    def broadcast_relay(self, src: int, dst_tensors, src_tensors, nblocks: int = 8):
        """Relay broadcast (peer stores) from emulated rank `src` into every
        rank's symmetric tensors dst_tensors[r] (lists from ``empty``)."""
        from . import weights  # noqa: F401  (declares the native signature)

        R = self.world
        if not hasattr(self, "_relay_seq"):
            self._relay_seq = {}
        seq = self._relay_seq.get(src, 0) + 1
        self._relay_seq[src] = seq
        keep, ptrs = [], []
        for r in range(R):
            base = self._lib.lz_emu_heap_ptr(self._emu, r)
            rows = []
            for i, d in enumerate(dst_tensors[r]):
                nbytes = d.numel() * d.element_size()
                srcp = src_tensors[i].data_ptr() if r == src else 0
                rows.append([srcp, d.data_ptr() - base, nbytes, 0])
            t = torch.tensor(rows, dtype=torch.int64, device=f"cuda:{self.device}")
            keep.append(t)
            ptrs.append(t.data_ptr())
        arr = (C.c_void_p * R)(*ptrs)
        rc = self._lib.lz_emu_weight_broadcast_relay(self._emu, src, arr, len(dst_tensors[0]), nblocks, seq,
                                                     torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "emulated relay broadcast")

    def status(self, r: int) -> int:
        return self._lib.lz_emu_status(self._emu, r)

    def close(self):
        if self._emu:
            self._lib.lz_emu_destroy(self._emu)
            self._emu = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
