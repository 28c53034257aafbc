"""All-to-all over NVLink peer memory, raw or with lossless compression.

    out = lz.all_to_all(x)                 # x: W equal chunks, chunk j -> rank j
    out = lz.all_to_all(x, compress=True)  # split + rANS records on the wire

One persistent launch per call (``csrc/lz_alltoall.cu``): raw chunks are
stored straight into the destination's output when that output is a
symmetric tensor (``comm.empty``), otherwise into its receive slot; the
compressed path encodes every 32768-element table group on the sender and
writes only the record into the destination's slot, which decodes it.

Reference behaviour: the compressed (LZip-NCCL) all-to-all compared with NCCL
in plot/cccl_alltoall.py:7-16, and the all-to-all exchange inside the
compressed two-shot allreduce
(single_node_nccl_allreduce_benchmark/compressed_twoshot_allreduce.py:148-163).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .. import _native, _native_sigs
from ..utils.dtypes import lz_dtype
from ..utils.trace import traced

_native_sigs.add_cuda({
    "lz_all_to_all": (C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int,
                      C.c_void_p),
    "lz_all_to_all_stage_bytes": (C.c_size_t, C.c_size_t, C.c_int, C.c_int, C.c_int),
    "lz_emu_all_to_all": (C.c_int, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_size_t,
                          C.c_int, C.c_int, C.c_int, C.c_void_p),
})

COMPRESSIBLE = (torch.bfloat16, torch.float16, torch.float32)


def stage_bytes_needed(numel: int, dtype: torch.dtype, world: int, compress: bool) -> int:
    """Stage bytes a call on `numel` elements (all chunks) needs."""
    return _native.cuda().lz_all_to_all_stage_bytes(numel // world, lz_dtype(dtype), world, int(compress))


def enc_code(compress) -> int:
    """Kernel encode code of the ``compress`` argument: False -> 0 (raw),
    True or "ans" -> 1 (split + rANS), "pack" -> 2 (split + PACK codes)."""
    if compress is False or compress is None or compress == 0:
        return 0
    if compress is True or compress == "ans" or compress == 1:
        return 1
    if compress == "pack":
        return 2
    raise ValueError(f"compress must be False, True, 'ans' or 'pack' (got {compress!r})")


@traced("all_to_all")
def all_to_all(x: torch.Tensor, out: torch.Tensor | None = None, compress: bool = False, comm=None,
               nblocks: int = 0, stream=None) -> torch.Tensor:
    """Exchange equal chunks: chunk j of every rank's ``x`` lands as chunk
    ``rank`` of rank j's output. CPU tensors go through ``dist.all_to_all_single``
    (``compress=True``: LZC1 streams of the CPU codec, sizes exchanged first).
    ``compress``: False, True / "ans" (split + rANS records) or "pack"
    (split + PACK table codes: faster codec, lower ratio)."""
    if not x.is_cuda:
        res = torch.empty_like(x) if out is None else out
        if enc_code(compress):
            return _all_to_all_compressed_cpu(x.contiguous(), res, level="pack" if compress == "pack" else "ans")
        dist.all_to_all_single(res, x.contiguous())
        return res
    from .allreduce import get_comm, init

    comm = comm or get_comm() or init()
    if not x.is_contiguous():
        raise ValueError("all_to_all needs a contiguous input")
    if x.numel() % comm.world:
        raise ValueError(f"{x.numel()} elements do not split into {comm.world} equal chunks")
    if compress and x.dtype not in COMPRESSIBLE:
        raise ValueError(f"compressed all_to_all supports {COMPRESSIBLE}, got {x.dtype}")
    if out is None:
        out = torch.empty_like(x)
    elif out.numel() != x.numel() or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor like x")
    dt = lz_dtype(x.dtype) if x.dtype in COMPRESSIBLE else 3  # raw: bytes
    chunk = x.numel() // comm.world
    if dt == 3:
        chunk *= x.element_size()
    s = stream or torch.cuda.current_stream(comm.device)
    rc = comm._lib.lz_all_to_all(comm.handle, x.data_ptr(), out.data_ptr(), chunk, dt, enc_code(compress),
                                 nblocks, s.cuda_stream)
    _native.check(rc, "all_to_all")
    return out


def _all_to_all_compressed_cpu(x: torch.Tensor, out: torch.Tensor, group=None, level="ans") -> torch.Tensor:
    """Host-side compressed all-to-all over any backend: every chunk is
    encoded with the CPU codec, the stream sizes are exchanged, then the
    streams (padded to the largest) and each received stream is decoded into
    its place. Lossless: the result equals the raw all-to-all bit for bit."""
    from ..ops import codec

    world = dist.get_world_size(group)
    if x.numel() % world:
        raise ValueError(f"{x.numel()} elements do not split into {world} equal chunks")
    if x.dtype not in COMPRESSIBLE:
        raise ValueError(f"compressed all_to_all supports {COMPRESSIBLE}, got {x.dtype}")
    chunks = x.view(world, -1)
    blobs = [codec.encode_cpu(chunks[j], level) for j in range(world)]
    sizes = torch.tensor([b.numel() for b in blobs], dtype=torch.int64)
    got_sizes = torch.empty_like(sizes)
    dist.all_to_all_single(got_sizes, sizes, group=group)
    cap_t = sizes.max().reshape(1)
    dist.all_reduce(cap_t, op=dist.ReduceOp.MAX, group=group)  # one padded size on every rank
    cap = int(cap_t.item())
    send = torch.zeros(world, cap, dtype=torch.uint8)
    for j, b in enumerate(blobs):
        send[j, : b.numel()] = b
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    o = out.view(world, -1)
    for j in range(world):
        o[j].copy_(codec.decode_cpu(recv[j, : int(got_sizes[j])], o.shape[1], x.dtype))
    return out

