"""Lossless compressed allreduce.

* :func:`compressed_allreduce` -- the native fused kernel (csrc/lz_compressed.cu):
  split+rANS encode fused with the peer push, decode fused with the fp32
  rank-order reduce, reduced slice re-encoded once and published with NVLS
  multimem.st. Bit-identical to an fp32 sequential reference.
* host-orchestrated variants over torch.distributed send/recv (any backend;
  CPU tensors use the CPU oracle codec, CUDA tensors the GPU codec):

  ==========================  ===========================================================
  ``compressed_twoshot``      all-to-all RS of compressed chunks, sum, compressed AG
                              ("LZip two-shot", single_node_nccl_allreduce_benchmark/
                              compressed_twoshot_allreduce.py:126-247)
  ``compressed_ring``         ring RS/AG, compression of the next chunk overlapping the
                              transfer of the current one
                              (single_node_nccl_allreduce_benchmark/compressed_sendrecv_allreduce.py:41-231)
  ``compressed_nosize``       two ranks, fixed-ratio budget, no size exchange
                              (single_node_nccl_allreduce_benchmark/compressed_nosize_allreduce.py:35-177)
  ``compressed_sizeexchange`` two ranks, exact sizes exchanged first
                              (back_up_nccl_allreduce_benchmark/compressed_sendrecv_allreduce.py:112-155)
  ==========================  ===========================================================

  The reference sends a fixed ``COMP_RATIO`` prefix and silently truncates
  streams that do not fit. Here every message is a fixed budget
  ``[u64 size | u64 flag | payload]``; a stream larger than the budget sends
  its remainder in a second message announced by the flag, so nothing is ever
  truncated, and the reported ratio is measured, not assumed.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .. import _native, _native_sigs
from ..ops import codec
from ..utils.dtypes import lz_dtype
from ..utils.trace import traced

_native_sigs.add_cuda({
    "lz_cz_stage_bytes": (C.c_size_t, C.c_size_t, C.c_int, C.c_int, C.c_int),
    "lz_cz_default_blocks": (C.c_int, C.c_void_p),
    "lz_compressed_allreduce": (C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_int,
                                C.c_int, C.c_void_p),
    "lz_emu_compressed_allreduce": (C.c_int, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                    C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_void_p),
    "lz_cz_stage_bytes_chunked": (C.c_size_t, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_size_t),
    "lz_cz_trace_slots": (C.c_int,),
    "lz_emu_compressed_allreduce_traced": (C.c_int, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                           C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p,
                                           C.c_void_p),
    "lz_compressed_allreduce_traced": (C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                       C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_void_p),
    "lz_compressed_allreduce_chunked": (C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                        C.c_int, C.c_int, C.c_size_t, C.c_void_p),
    "lz_emu_compressed_allreduce_chunked": (C.c_int, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                            C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p),
})

HDR = 16  # u64 stream size + u64 overflow flag


# ----------------------------------------------------------------------------- native
# Phases of the per-CTA tracer of the native kernel (csrc/lz_compressed.cu CzPhase).
TRACE_PHASES = ("total", "start_barrier", "rs_encode_push", "rs_wait", "rs_decode", "reduce", "ag_encode",
                "ag_push", "ag_wait", "ag_decode", "chunk_wait", "tgs_reduced")


# Default chunk of large calls. Measured with 1 GiB bf16 per rank: 2 x B200,
# hybrid PACK 1.96 ms with 256 MB chunks vs 2.17 ms in one chunk (fully
# compressed PACK 2.13 vs 2.23); 8 x B200, hybrid PACK 3.74 vs 4.20 ms. The
# chunk also bounds the stage memory to two chunks' slots.
AUTO_CHUNK_BYTES = 256 << 20


def trace_buffer(comm=None, nblocks: int = 0) -> torch.Tensor:
    """Zeroed tracer rows (int64, one per CTA) for compressed_allreduce(trace=)."""
    from .allreduce import get_comm

    comm = comm or get_comm()
    g = nblocks or comm.config.sm_budget or comm._lib.lz_cz_default_blocks(comm.handle)
    assert comm._lib.lz_cz_trace_slots() == len(TRACE_PHASES)
    return torch.zeros((g, len(TRACE_PHASES)), dtype=torch.int64, device=f"cuda:{comm.device}")


def summarize_trace(buf: torch.Tensor, calls: int = 1) -> dict:
    """Mean microseconds per CTA and call for every phase (the last entry is
    table groups reduced per CTA and call)."""
    m = buf.double().mean(dim=0).cpu() / max(calls, 1)
    return {name: (round(float(v) / 1e3, 2) if name != "tgs_reduced" else round(float(v), 2))
            for name, v in zip(TRACE_PHASES, m)}


def stage_bytes_needed(n: int, dtype: torch.dtype, world: int, nblocks: int = 444, chunk_elems: int = 0) -> int:
    """Stage bytes of a native compressed allreduce of n elements; with
    ``chunk_elems`` > 0 the call runs in chunks of that many elements and
    needs slots for two chunks only."""
    return int(_native.cuda().lz_cz_stage_bytes_chunked(n, lz_dtype(dtype), world, nblocks, chunk_elems))


@traced("compressed_allreduce")
def compressed_allreduce(t: torch.Tensor, out: torch.Tensor | None = None, comm=None,
                         nblocks: int = 0, multicast: bool = True, stream=None,
                         hybrid: bool = False, level="ans", chunk_bytes: int | None = None,
                         stage_local: bool = False, trace: torch.Tensor | None = None) -> torch.Tensor:
    """Sum-allreduce with lossless compression on the wire (native fused kernel).

    ``level``: codec level of the records, "ans" (rANS, best ratio) or "pack"
    (table codes: a few integer operations per element, ratio ~0.70 for bf16
    instead of ~0.67).

    ``chunk_bytes`` (default: :data:`AUTO_CHUNK_BYTES` for vectors larger than
    that, else one chunk; 0 forces one chunk) > 0 processes the vector in chunks of that many bytes
    inside the one launch: every slice moves chunk by chunk through a ring of
    two chunks' slots, so the stage memory is bounded by the chunk size while
    encoding, transfer and decoding of neighbouring chunks overlap (a CTA
    starts chunk k + 2 as soon as every rank's same CTA has finished chunk k).
    ``stage_local`` encodes reduce-scatter records next to the encoding CTA
    and pushes them to the peer in 16-byte vectors instead of encoding
    straight into the peer's slot.
    ``trace``: an int64 CUDA tensor from :func:`trace_buffer`; every CTA adds
    the nanoseconds it spent in each phase (:data:`TRACE_PHASES`) to its row
    (read with :func:`summarize_trace`).

    ``hybrid=True`` is the compressed P2P hybrid: the reduce-scatter moves raw
    bytes and only the all-gather of the reduced slices is compressed, so each
    GPU encodes 1/W of the vector instead of all of it
    (single_node_nccl_allreduce_benchmark/compressed_p2p_allreduce.py:54-188 of the reference).
    """
    from .allreduce import get_comm, init

    if not t.is_cuda:
        return compressed_twoshot(t)
    comm = comm or get_comm() or init()
    if out is None:
        out = t
    s = stream or torch.cuda.current_stream(comm.device)
    nb = nblocks or comm.config.sm_budget
    if chunk_bytes is None:
        chunk_bytes = AUTO_CHUNK_BYTES if t.numel() * t.element_size() > AUTO_CHUNK_BYTES else 0
    chunk_elems = chunk_bytes // t.element_size() if chunk_bytes else 0
    if trace is not None and (trace.dtype != torch.int64 or not trace.is_cuda or
                              trace.numel() < (nb or comm._lib.lz_cz_default_blocks(comm.handle)) * len(TRACE_PHASES)):
        raise ValueError("trace must be the int64 CUDA tensor of trace_buffer(comm, nblocks)")
    rc = comm._lib.lz_compressed_allreduce_traced(comm.handle, t.data_ptr(), out.data_ptr(), t.numel(),
                                                  lz_dtype(t.dtype), nb,
                                                  int(multicast) | (2 if hybrid else 0) |
                                                  (4 * codec.level_code(level)) | (8 if stage_local else 0),
                                                  chunk_elems, trace.data_ptr() if trace is not None else None,
                                                  s.cuda_stream)
    _native.check(rc, "compressed_allreduce")
    return out


# ----------------------------------------------------------------------------- messages
@traced("compress")
def _encode(x: torch.Tensor) -> torch.Tensor:
    return codec.encode(x) if x.is_cuda else codec.encode_cpu(x)


@traced("decompress")
def _decode(blob: torch.Tensor, n: int, dtype, out: torch.Tensor | None = None) -> torch.Tensor:
    y = codec.decode(blob, n=n, dtype=dtype) if blob.is_cuda else codec.decode_cpu(blob, n, dtype)
    if out is not None:
        out.copy_(y.view(out.shape))
        return out
    return y


def budget_bytes(numel: int, elem: int, ratio: float) -> int:
    """Fixed message size for a chunk at an assumed compression ratio."""
    b = int(numel * elem * ratio) + HDR
    return (b + 15) // 16 * 16


def _pack(blob: torch.Tensor, budget: int):
    """-> (fixed message, optional overflow remainder)."""
    size = blob.numel()
    msg = torch.zeros(budget, dtype=torch.uint8, device=blob.device)
    room = budget - HDR
    over = size > room
    hdr = torch.tensor([size, int(over)], dtype=torch.int64)
    msg[:HDR].copy_(hdr.view(torch.uint8))
    msg[HDR:HDR + min(size, room)].copy_(blob[:room])
    rest = blob[room:].contiguous() if over else None
    return msg, rest


def _unpack_header(msg: torch.Tensor):
    hdr = msg[:HDR].cpu().view(torch.int64)
    return int(hdr[0]), bool(hdr[1])


class _Stats:
    def __init__(self):
        self.raw_bytes = 0
        self.sent_bytes = 0
        self.overflows = 0

    @property
    def ratio(self):
        return self.sent_bytes / self.raw_bytes if self.raw_bytes else float("nan")


STATS = _Stats()


@traced("exchange")
def _exchange_compressed(pairs, group, budget):
    """pairs: list of (peer, blob_to_send, (n, dtype, out_or_None)) -> decoded list.

    Phase 1: fixed-budget messages both ways; phase 2: overflow remainders.
    """
    sends, recvs, ops = [], [], []
    for peer, blob, _ in pairs:
        msg, rest = _pack(blob, budget)
        sends.append(rest)
        r = torch.empty(budget, dtype=torch.uint8, device=blob.device)
        recvs.append(r)
        ops.append(dist.P2POp(dist.isend, msg, peer, group=group))
        ops.append(dist.P2POp(dist.irecv, r, peer, group=group))
        STATS.sent_bytes += min(blob.numel(), budget - HDR) + HDR
    for w in dist.batch_isend_irecv(ops):
        w.wait()
    ops2, tails = [], []
    for (peer, blob, _), rest, r in zip(pairs, sends, recvs):
        size, over = _unpack_header(r)
        tail = None
        if rest is not None:
            ops2.append(dist.P2POp(dist.isend, rest, peer, group=group))
            STATS.sent_bytes += rest.numel()
            STATS.overflows += 1
        if over:
            tail = torch.empty(size - (budget - HDR), dtype=torch.uint8, device=r.device)
            ops2.append(dist.P2POp(dist.irecv, tail, peer, group=group))
        tails.append((size, tail))
    if ops2:
        for w in dist.batch_isend_irecv(ops2):
            w.wait()
    out = []
    for (peer, blob, (n, dtype, dst)), r, (size, tail) in zip(pairs, recvs, tails):
        stream = r[HDR:HDR + min(size, budget - HDR)]
        if tail is not None:
            stream = torch.cat([stream, tail])
        out.append(_decode(stream.contiguous(), n, dtype, dst))
    return out


def _info(group):
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(ws))
    return rank, ws, ranks


def _chunks(t, ws):
    n = t.numel()
    base = n // ws
    return [t[i * base: (n if i == ws - 1 else (i + 1) * base)] for i in range(ws)]


# ----------------------------------------------------------------------------- variants
def compressed_twoshot(t: torch.Tensor, group=None, ratio: float = 0.65) -> torch.Tensor:
    """All-to-all RS of compressed chunks, fp32 rank-order sum, compressed AG."""
    rank, ws, gr = _info(group)
    if ws == 1:
        return t
    ch = _chunks(t, ws)
    budget = budget_bytes(max(c.numel() for c in ch), t.element_size(), ratio)
    pairs = []
    for p in range(ws):
        if p != rank:
            pairs.append((gr[p], _encode(ch[p].contiguous()), (ch[rank].numel(), t.dtype, None)))
            STATS.raw_bytes += ch[p].numel() * t.element_size()
    got = _exchange_compressed(pairs, group, budget)
    others = iter(got)
    acc = None
    for p in range(ws):  # rank order, fp32
        v = ch[rank] if p == rank else next(others).view(ch[rank].shape)
        acc = v.float().clone() if acc is None else acc + v.float()
    ch[rank].copy_(acc)
    mine = _encode(ch[rank].contiguous())
    pairs = []
    for p in range(ws):
        if p != rank:
            pairs.append((gr[p], mine, (ch[p].numel(), t.dtype, ch[p])))
            STATS.raw_bytes += ch[rank].numel() * t.element_size()
    _exchange_compressed(pairs, group, budget)
    return t


def compressed_ring(t: torch.Tensor, group=None, ratio: float = 0.65, pieces: int = 2) -> torch.Tensor:
    """Ring RS + AG over compressed chunks (bf16 partial sums per hop, as NCCL).

    Double-buffered: every ring chunk travels as ``pieces`` pieces whose
    fixed-budget messages are posted asynchronously (isend/irecv), so piece
    k + 1 is encoded while piece k is on the wire; received pieces are decoded
    after the posts. The all-gather forwards the compressed stream it received
    instead of re-encoding it. The reference overlaps compression of the next
    chunk with the current transfer in the same way
    (single_node_nccl_allreduce_benchmark/compressed_sendrecv_allreduce.py:41-231).
    """
    rank, ws, gr = _info(group)
    if ws == 1:
        return t
    ch = _chunks(t, ws)
    right, left = gr[(rank + 1) % ws], gr[(rank - 1) % ws]
    P = max(1, int(pieces))

    def parts(x):  # P contiguous pieces of a chunk view
        n = x.numel()
        return [x[(n * k) // P:(n * (k + 1)) // P] for k in range(P)]

    pbudget = budget_bytes(max(c.numel() for c in ch) // P + 1, t.element_size(), ratio)

    def hop(send_blobs, recv_shapes, encode_next=None):
        """One ring step: post every piece's message (encoding the next piece
        while the previous one is in flight), then finish overflows and return
        the received streams (compressed, per piece)."""
        posted = []
        blob = send_blobs(0)
        for k in range(P):
            msg, rest = _pack(blob, pbudget)
            r = torch.empty(pbudget, dtype=torch.uint8, device=t.device)
            works = dist.batch_isend_irecv([dist.P2POp(dist.isend, msg, right, group=group),
                                            dist.P2POp(dist.irecv, r, left, group=group)])
            STATS.sent_bytes += min(blob.numel(), pbudget - HDR) + HDR
            posted.append((works, msg, r, rest))
            if k + 1 < P:
                blob = send_blobs(k + 1)  # overlaps the transfer of piece k
        streams = []
        for works, msg, r, rest in posted:
            for w in works:
                w.wait()
            size, over = _unpack_header(r)
            ops, tail = [], None
            if rest is not None:
                ops.append(dist.P2POp(dist.isend, rest, right, group=group))
                STATS.sent_bytes += rest.numel()
                STATS.overflows += 1
            if over:
                tail = torch.empty(size - (pbudget - HDR), dtype=torch.uint8, device=r.device)
                ops.append(dist.P2POp(dist.irecv, tail, left, group=group))
            if ops:
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
            stream = r[HDR:HDR + min(size, pbudget - HDR)]
            streams.append(torch.cat([stream, tail]) if tail is not None else stream.contiguous())
        return streams

    # reduce-scatter: send my partial sum of chunk si, add the received one into chunk ri
    si, ri = rank, (rank - 1) % ws
    for _ in range(ws - 1):
        src_parts, dst_parts = parts(ch[si]), parts(ch[ri])
        got = hop(lambda k, sp=src_parts: _encode(sp[k].contiguous()), None)
        for k, g in enumerate(got):
            dst_parts[k].add_(_decode(g, dst_parts[k].numel(), t.dtype).view(dst_parts[k].shape))
        STATS.raw_bytes += ch[si].numel() * t.element_size()
        si, ri = ri, (ri - 1) % ws
    # all-gather: encode my reduced chunk once, then forward what arrives
    si, ri = (rank + 1) % ws, rank
    fwd = [_encode(x.contiguous()) for x in parts(ch[si])]
    for _ in range(ws - 1):
        got = hop(lambda k, f=fwd: f[k], None)
        dst_parts = parts(ch[ri])
        for k, g in enumerate(got):
            dst_parts[k].copy_(_decode(g, dst_parts[k].numel(), t.dtype).view(dst_parts[k].shape))
        STATS.raw_bytes += ch[si].numel() * t.element_size()
        fwd = got
        si, ri = ri, (ri - 1) % ws
    return t


def compressed_nosize(t: torch.Tensor, group=None, ratio: float = 0.65) -> torch.Tensor:
    rank, ws, _ = _info(group)
    if ws != 2:
        raise ValueError("compressed_nosize is a two-rank algorithm")
    return compressed_twoshot(t, group, ratio)


def compressed_sizeexchange(t: torch.Tensor, group=None) -> torch.Tensor:
    """Two ranks: exchange exact compressed sizes first, then the streams."""
    rank, ws, gr = _info(group)
    if ws != 2:
        raise ValueError("compressed_sizeexchange is a two-rank algorithm")
    peer = gr[1 - rank]
    ch = _chunks(t, 2)

    def swap(blob, n_recv, dst):
        mine = torch.tensor([blob.numel()], dtype=torch.int64, device=blob.device)
        theirs = torch.empty_like(mine)
        for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, mine, peer, group=group),
                                         dist.P2POp(dist.irecv, theirs, peer, group=group)]):
            w.wait()
        r = torch.empty(int(theirs.item()), dtype=torch.uint8, device=blob.device)
        for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, blob, peer, group=group),
                                         dist.P2POp(dist.irecv, r, peer, group=group)]):
            w.wait()
        STATS.sent_bytes += blob.numel() + 8
        return _decode(r, n_recv, t.dtype, dst)

    other = swap(_encode(ch[1 - rank].contiguous()), ch[rank].numel(), None).view(ch[rank].shape)
    STATS.raw_bytes += ch[1 - rank].numel() * t.element_size()
    acc = (ch[0].float() + other.float()) if rank == 0 else (other.float() + ch[1].float())
    ch[rank].copy_(acc)
    swap(_encode(ch[rank].contiguous()), ch[1 - rank].numel(), ch[1 - rank])
    STATS.raw_bytes += ch[rank].numel() * t.element_size()
    return t


VARIANTS = {
    "compressed_twoshot": compressed_twoshot,
    "compressed_ring": compressed_ring,
    "compressed_nosize": compressed_nosize,
    "compressed_sizeexchange": compressed_sizeexchange,
}
