"""RL weight-update transfer (trainer rank -> inference ranks).

B200 design: one persistent kernel per bucket and rank (csrc/lz_weights.cu).
Table groups of 32K elements are split + rANS encoded by the sender (or sent
raw) into K slots per CTA on every receiver and decoded there straight into
the destination tensors, chunk-pipelined with credits. When every other rank
receives, records go out with NVLS multimem.st: the switch replicates one
write to all receivers, so the sender's link carries each byte once.

Public API::

    wt = WeightTransfer(comm, mode="split_ans")      # or "raw"
    wt.send(tensors, dsts=[1, 2])     # trainer
    wt.recv(tensors, src=0)           # each receiver (destination tensors, same shapes)
    wt.broadcast(tensors, src=0)      # all ranks; src sends, others receive
    send_weights(state_dict, dst) / recv_weights(state_dict, src) / broadcast_weights(sd, src)

Reference counterpart: UpdateWeightFromDistributed
(back_up/update_weight_from_distributed.py:37-376): buckets by
``update_weight_buffer_size`` (:259), per-tensor NCCL broadcast (:422-449),
optional safetensors dump with a JSONL manifest (:93-160).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import time
import weakref

import torch
import torch.distributed as dist

from .. import _native, _native_sigs
from ..ops import codec
from ..utils import trace

_native_sigs.add_cuda({
    "lz_wx_slot_capacity": (C.c_size_t,),
    "lz_wx_tg_elems": (C.c_size_t,),
    "lz_wx_stage_bytes": (C.c_size_t, C.c_int, C.c_int),
    "lz_wx_group": (C.c_int,),
    "lz_weight_transfer": (C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_uint, C.c_void_p, C.c_uint, C.c_int,
                           C.c_int, C.c_int, C.POINTER(C.c_uint64), C.c_void_p),
    "lz_weight_transfer_direct": (C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_uint, C.c_void_p, C.c_uint,
                                  C.c_int, C.c_int, C.POINTER(C.c_uint64), C.c_void_p),
    "lz_weight_broadcast_relay": (C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_uint, C.c_int, C.c_int,
                                  C.c_uint64, C.c_void_p),
    "lz_emu_weight_broadcast_relay": (C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_void_p), C.c_uint, C.c_int,
                                      C.c_uint64, C.c_void_p),
    "lz_weight_transfer_ce": (C.c_int, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_uint64),
                              C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.c_uint, C.c_uint64, C.c_void_p),
})

TG = 32768
MODES = ("raw", "split_ans", "split_pack")
# descriptor encode field per mode: 0 raw, 1 split + rANS, 2 split + PACK codes
_ENCODE_CODE = {"raw": 0, "split_ans": 1, "split_pack": 2}


def _encode_flags(n_tensors: int, fraction: float):
    """Evenly spread selection of round(fraction * n) tensors to encode."""
    return [int((i + 1) * fraction) > int(i * fraction) for i in range(n_tensors)]


def build_descriptors(tensors, encode, device) -> tuple[torch.Tensor, int]:
    """16-byte descriptor per table group: (ptr, n | dtype << 32 | encode << 40),
    encode = 0 (raw), 1 (split + rANS, also for True) or 2 (split + PACK codes)."""
    rows_ptr, rows_meta = [], []
    for t, enc in zip(tensors, encode):
        if not t.is_contiguous():
            raise ValueError("weight transfer needs contiguous tensors")
        if t.numel() == 0:
            continue
        base = t.data_ptr()
        if base % 16:
            raise ValueError("weight transfer needs 16-byte aligned tensors")
        # fp8 tensors of even length travel as packed pairs (fused pack/unpack)
        dt, numel = codec.plan(t.dtype, t.numel())
        es = 4 if dt == 0 else (1 if dt == 3 else 2)
        ntg = (numel + TG - 1) // TG
        idx = torch.arange(ntg, dtype=torch.int64)
        rows_ptr.append(base + idx * (TG * es))
        n = torch.clamp(numel - idx * TG, max=TG)
        code = int(enc)
        if code not in (0, 1, 2):
            raise ValueError(f"encode code {enc!r} must be 0, 1 or 2")
        rows_meta.append(n | (dt << 32) | (code << 40))
    if not rows_ptr:
        return torch.empty(0, dtype=torch.int64, device=device), 0
    d = torch.stack([torch.cat(rows_ptr), torch.cat(rows_meta)], dim=1).contiguous()
    return d.pin_memory().to(device, non_blocking=True), d.shape[0]


class WeightTransfer:
    """Chunk-pipelined weight transfer engine on a :class:`Communicator`."""

    def __init__(self, comm, mode: str = "split_ans", nblocks: int = 0, kslots: int = 0,
                 chunk_bytes: int = 0, encode_fraction: float = 1.0):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        self.comm = comm
        self.mode = mode
        self.encode_fraction = encode_fraction if mode != "raw" else 0.0
        self.nblocks = nblocks or comm.sm_count * 2
        cap_tg_bytes = TG * 2
        if kslots:
            self.kslots = kslots
        elif chunk_bytes:
            self.kslots = max(2, chunk_bytes // (self.nblocks * cap_tg_bytes))
        else:
            self.kslots = 4
        lib = comm._lib
        grp = lib.lz_wx_group()
        need = lib.lz_wx_stage_bytes(self.nblocks, self.kslots) * grp
        if need > comm.config.stage_bytes:
            self.kslots = max(2, comm.config.stage_bytes // (self.nblocks * lib.lz_wx_slot_capacity() * grp))
            if lib.lz_wx_stage_bytes(self.nblocks, self.kslots) * grp > comm.config.stage_bytes:
                self.nblocks = max(1, comm.config.stage_bytes // (2 * lib.lz_wx_slot_capacity() * grp))
        # Flag sequence numbers must be monotonic per communicator (not per
        # engine): every engine on `comm` shares the same flag words.
        if not hasattr(comm, "_wx_pair_seq"):
            comm._wx_pair_seq = {}
            comm._wx_bcast_seq = {}
        self.pair_seq: dict = comm._wx_pair_seq
        self.bcast_seq: dict = comm._wx_bcast_seq
        self.bytes_sent = 0

    @property
    def window_bytes(self) -> int:
        """Bytes in flight: blocks x slots x one table group of bf16."""
        return self.nblocks * self.kslots * TG * 2

    def _launch(self, role, src, mask, descs, ntg, all_, seqs):
        arr = (C.c_uint64 * 8)(*seqs)
        s = torch.cuda.current_stream(self.comm.device)
        # flags: bit 0 every other rank receives, bit 1 records at the codec's PACK level
        flags = int(all_) | (2 if self.mode == "split_pack" else 0)
        rc = self.comm._lib.lz_weight_transfer(self.comm.handle, role, src, mask, descs.data_ptr(), ntg,
                                               self.nblocks, self.kslots, flags, arr, s.cuda_stream)
        _native.check(rc, "weight transfer")

    def _flags(self, tensors):
        f = self.encode_fraction
        code = _ENCODE_CODE[self.mode]
        return [code if e else 0 for e in _encode_flags(len(tensors), f)] if f > 0 else [0] * len(tensors)

    def send(self, tensors, dsts, broadcast_all: bool = False) -> None:
        tensors = list(tensors.values()) if isinstance(tensors, dict) else list(tensors)
        dsts = [dsts] if isinstance(dsts, int) else list(dsts)
        me = self.comm.rank
        mask = 0
        for d in dsts:
            mask |= 1 << d
        descs, ntg = build_descriptors(tensors, self._flags(tensors), f"cuda:{self.comm.device}")
        seqs = [0] * 8
        if broadcast_all:
            s = self.bcast_seq.get(me, 0) + 1
            self.bcast_seq[me] = s
            seqs = [s] * 8
        else:
            for d in dsts:
                s = self.pair_seq.get((me, d), 0) + 1
                self.pair_seq[(me, d)] = s
                seqs[d] = s
        self.bytes_sent += sum(t.numel() * t.element_size() for t in tensors)
        self._launch(0, me, mask, descs, ntg, broadcast_all, seqs)
        self._keep = descs  # descriptors must outlive the launch

    def recv(self, tensors, src: int, broadcast_all: bool = False) -> None:
        tensors = list(tensors.values()) if isinstance(tensors, dict) else list(tensors)
        me = self.comm.rank
        descs, ntg = build_descriptors(tensors, self._flags(tensors), f"cuda:{self.comm.device}")
        if broadcast_all:
            s = self.bcast_seq.get(src, 0) + 1
            self.bcast_seq[src] = s
            mask = ((1 << self.comm.world) - 1) & ~(1 << src)
        else:
            s = self.pair_seq.get((src, me), 0) + 1
            self.pair_seq[(src, me)] = s
            mask = 1 << me
        self._launch(1, src, mask, descs, ntg, broadcast_all, [s] * 8)
        self._keep = descs

    # ------------------------------------------------------------ zero-copy raw
    def _direct_descs(self, dst_tensors, src_tensors):
        comm = self.comm
        rows = []
        for i, d in enumerate(dst_tensors):
            if not comm.is_symmetric(d):
                raise ValueError("direct transfer needs destination tensors allocated with comm.empty()")
            srcp = src_tensors[i].data_ptr() if src_tensors is not None else 0
            if src_tensors is not None and (src_tensors[i].numel() * src_tensors[i].element_size()
                                            != d.numel() * d.element_size()):
                raise ValueError("source and destination sizes differ")
            rows.append([srcp, d.data_ptr() - comm._local_base, d.numel() * d.element_size(), 0])
        t = torch.tensor(rows, dtype=torch.int64).pin_memory()
        return t.to(f"cuda:{comm.device}", non_blocking=True), len(rows)

    def send_copy_engine(self, dst_tensors, src: int, dst: int, src_tensors=None) -> None:
        """Zero-copy point-to-point transfer by DMA: rank `src` copies its
        ``src_tensors`` (default: its own ``dst_tensors``) into rank `dst`'s
        symmetric ``dst_tensors`` with the copy engines (no SM does the data
        movement). Both ranks call; other ranks do nothing."""
        comm = self.comm
        me = comm.rank
        if me not in (src, dst) or src == dst:
            return
        key = (src, dst)
        s = self.pair_seq.get(key, 0) + 1
        self.pair_seq[key] = s
        st = torch.cuda.current_stream(comm.device)
        n = len(dst_tensors)
        if me == src:
            srcs = src_tensors if src_tensors is not None else dst_tensors
            ptrs = (C.c_uint64 * n)(*[t.data_ptr() for t in srcs])
            offs, sizes = [], []
            for t_s, t_d in zip(srcs, dst_tensors):
                if not comm.is_symmetric(t_d):
                    raise ValueError("copy-engine transfer needs destination tensors allocated with comm.empty()")
                nb = t_d.numel() * t_d.element_size()
                if t_s.numel() * t_s.element_size() != nb:
                    raise ValueError("source and destination sizes differ")
                offs.append(t_d.data_ptr() - comm._local_base)
                sizes.append(nb)
            rc = comm._lib.lz_weight_transfer_ce(comm.handle, 0, dst, ptrs, (C.c_uint64 * n)(*offs),
                                                 (C.c_uint64 * n)(*sizes), n, s, st.cuda_stream)
        else:
            rc = comm._lib.lz_weight_transfer_ce(comm.handle, 1, src, None, None, None, 0, s, st.cuda_stream)
        _native.check(rc, "copy-engine transfer")

    def broadcast_direct(self, dst_tensors, src: int, src_tensors=None, nblocks: int = 0,
                         relay: bool | None = None, copy_engine: bool | None = None) -> None:
        """Zero-copy raw broadcast into symmetric destination tensors.

        Every rank passes its symmetric destination tensors (allocated with
        ``comm.empty`` in the same order on all ranks); the sender also passes
        ``src_tensors`` (default: its own destination tensors).

        Two ranks with tensors of 16 MB and more on average (``copy_engine``
        default): the copy engines move the bytes (765 GB/s for 1 GB on
        2 x B200, vs 643 GB/s for SM peer stores); smaller tensors use the
        one-launch peer-store kernel.
        More than two ranks (``relay`` default): the sender hands each 256 KB
        chunk to one owner rank, which forwards it to every other rank
        (multimem.st through the switch when multicast is available), so all
        GPUs' NVLink egress carries the broadcast and every receiver takes in
        each byte once. ``relay=False, copy_engine=False``: the sender stores
        every chunk into every receiver itself.
        """
        comm = self.comm
        if comm.world == 1:
            if src_tensors is not None:
                for d, s_ in zip(dst_tensors, src_tensors):
                    d.copy_(s_)
            return
        if copy_engine is None:
            # copy engines pay a per-copy launch cost: use them for large tensors
            # (2 x B200: KV cache of 80 x 3.9 MB tensors 0.77 ms by DMA vs 0.57 ms by
            # SM stores; 80 x 52 MB 6.05 vs 6.40 ms; GLM-4-9B, 66 MB average, 26.9 vs 28.8 ms)
            nbytes = sum(t.numel() * t.element_size() for t in dst_tensors)
            copy_engine = comm.world == 2 and not relay and nbytes >= (16 << 20) * max(1, len(dst_tensors))
        if copy_engine:
            if comm.world != 2:
                raise ValueError("the copy-engine path is point to point (2 ranks); use relay for more")
            own = comm.rank == src and src_tensors is not None and any(
                d_.data_ptr() != s_.data_ptr() for d_, s_ in zip(dst_tensors, src_tensors))
            if own:
                # the sender's own destination copy (the kernel paths write it too),
                # on a side stream so it overlaps the DMA to the receiver
                cur = torch.cuda.current_stream(comm.device)
                side = self.__dict__.setdefault("_side", torch.cuda.Stream(comm.device))
                side.wait_stream(cur)
            self.send_copy_engine(dst_tensors, src, 1 - src, src_tensors=src_tensors)
            if own:
                with torch.cuda.stream(side):
                    for d_, s_ in zip(dst_tensors, src_tensors):
                        if d_.data_ptr() != s_.data_ptr():
                            d_.copy_(s_)
                cur.wait_stream(side)
            return
        me = comm.rank
        mask = ((1 << comm.world) - 1) & ~(1 << src)
        s = self.bcast_seq.get(src, 0) + 1
        self.bcast_seq[src] = s
        if relay is None:
            relay = comm.world > 2
        if relay:
            descs, nd = self._direct_descs(dst_tensors, (src_tensors if src_tensors is not None else dst_tensors)
                                           if me == src else None)
            st = torch.cuda.current_stream(comm.device)
            rc = comm._lib.lz_weight_broadcast_relay(comm.handle, src, descs.data_ptr(), nd,
                                                     nblocks or min(comm.sm_count * 2, 512),
                                                     int(comm.has_multicast), s, st.cuda_stream)
            _native.check(rc, "relay weight broadcast")
            self._keep = descs
            return
        if me == src:
            descs, nd = self._direct_descs(dst_tensors, src_tensors if src_tensors is not None else dst_tensors)
            role = 0
        else:
            descs, nd = self._direct_descs(dst_tensors, None)
            role = 1
        arr = (C.c_uint64 * 8)(*([s] * 8))
        st = torch.cuda.current_stream(comm.device)
        rc = comm._lib.lz_weight_transfer_direct(comm.handle, role, src, mask, descs.data_ptr(), nd,
                                                 nblocks or min(comm.sm_count * 2, 512), 1, arr, st.cuda_stream)
        _native.check(rc, "direct weight transfer")
        self._keep = descs

    def broadcast_staged(self, dst_tensors, src: int, src_tensors=None, stage_bytes: int = 256 << 20) -> None:
        """Raw broadcast into ANY destination tensors (not only symmetric ones).

        The bytes go through two symmetric staging buffers of ``stage_bytes``:
        bucket k is broadcast into buffer k mod 2 with :meth:`broadcast_direct`
        (relay broadcast with multicast forwarding for more than two ranks,
        copy engines at two), then every receiver copies it out into its own
        destination tensors on a side stream while bucket k+1 is broadcast
        into the other buffer. The broadcast of bucket k+2 waits for the
        copy-out of bucket k on every rank (stream order before the relay's
        start barrier). All ranks call with tensors of the same sizes, in the
        same order; the sender passes its sources as ``src_tensors`` (default:
        its ``dst_tensors``). Contiguous tensors only.
        """
        comm = self.comm
        if comm.world == 1:
            if src_tensors is not None:
                for d, s_ in zip(dst_tensors, src_tensors):
                    d.copy_(s_)
            return
        stage_bytes = max(1 << 20, (stage_bytes + 4095) // 4096 * 4096)
        st = self.__dict__.get("_stage")
        if st is None or st[0].numel() < stage_bytes:
            # collective: every rank allocates the same buffers in the same order
            st = [comm.empty(stage_bytes, torch.uint8), comm.empty(stage_bytes, torch.uint8)]
            self._stage = st
        cap = st[0].numel()
        me = comm.rank
        srcs = src_tensors if src_tensors is not None else dst_tensors
        # pieces: (tensor index, byte offset, bytes) packed into buckets of <= cap
        buckets, cur, used = [], [], 0
        for i, d in enumerate(dst_tensors):
            if not d.is_contiguous() or (me == src and not srcs[i].is_contiguous()):
                raise ValueError("broadcast_staged needs contiguous tensors")
            nb = d.numel() * d.element_size()
            off = 0
            while off < nb:
                room = cap - used
                if room < 4096:
                    buckets.append(cur)
                    cur, used = [], 0
                    room = cap
                take = min(nb - off, room // 16 * 16)
                cur.append((i, off, take, used))
                used = (used + take + 255) // 256 * 256
                off += take
        if cur:
            buckets.append(cur)
        cs = torch.cuda.current_stream(comm.device)
        side = self.__dict__.setdefault("_side", torch.cuda.Stream(comm.device))
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        sent = torch.cuda.Event()
        for k, bkt in enumerate(buckets):
            buf = st[k % 2]
            if k >= 2:
                cs.wait_event(copied[k % 2])
            views = [buf[so:so + n] for (_, _, n, so) in bkt]
            sviews = None
            if me == src:
                sviews = [srcs[i].view(-1).view(torch.uint8)[o:o + n] for (i, o, n, _) in bkt]
            self.broadcast_direct(views, src, sviews)
            sent.record(cs)
            side.wait_event(sent)
            with torch.cuda.stream(side):
                for (i, o, n, so), v in zip(bkt, views):
                    d = dst_tensors[i].view(-1).view(torch.uint8)[o:o + n]
                    if me != src or d.data_ptr() != srcs[i].view(-1).view(torch.uint8)[o:o + n].data_ptr():
                        d.copy_(v if me != src else srcs[i].view(-1).view(torch.uint8)[o:o + n])
                copied[k % 2].record(side)
        cs.wait_stream(side)

    def broadcast(self, tensors, src: int) -> None:
        """All ranks call; `src` sends its tensors, every other rank receives into its own."""
        others = [r for r in range(self.comm.world) if r != src]
        if self.comm.world == 1:
            return
        if self.comm.rank == src:
            self.send(tensors, others, broadcast_all=True)
        else:
            self.recv(tensors, src, broadcast_all=True)


# ---------------------------------------------------------------------- buckets
def buckets(named, max_bytes: int):
    """Group (name, tensor) pairs into buckets of at most `max_bytes` (one oversize tensor alone)."""
    cur, size = [], 0
    for name, t in named:
        nb = t.numel() * t.element_size()
        if cur and size + nb > max_bytes:
            yield cur
            cur, size = [], 0
        cur.append((name, t))
        size += nb
    if cur:
        yield cur


# ------------------------------------------------------------ host transport
class HostTransfer:
    """Weight transfer of CPU tensors over any torch.distributed backend
    (gloo): per tensor, raw bytes, or an LZC1 stream of the CPU codec with its
    size sent first (``split_ans`` / ``split_pack``). The same public calls (send / recv /
    broadcast) as :class:`WeightTransfer`; receivers end bit-identical."""

    def __init__(self, mode: str = "split_ans", group=None):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        self.mode, self.group = mode, group

    def _encode(self, t):
        if self.mode == "raw" or t.dtype not in _CODEC_DTYPES:
            return None
        return codec.encode_cpu(t, level="pack" if self.mode == "split_pack" else "ans")

    def send(self, tensors, dsts) -> None:
        dsts = [dsts] if isinstance(dsts, int) else list(dsts)
        for t in tensors:
            blob = self._encode(t)
            for d in dsts:
                if blob is None:
                    dist.send(t.contiguous(), d, group=self.group)
                else:
                    dist.send(torch.tensor([blob.numel()], dtype=torch.int64), d, group=self.group)
                    dist.send(blob, d, group=self.group)

    def recv(self, tensors, src: int) -> None:
        for t in tensors:
            if self.mode == "raw" or t.dtype not in _CODEC_DTYPES:
                buf = t if t.is_contiguous() else torch.empty_like(t)
                dist.recv(buf, src, group=self.group)
                if buf is not t:
                    t.copy_(buf)
                continue
            n = torch.empty(1, dtype=torch.int64)
            dist.recv(n, src, group=self.group)
            blob = torch.empty(int(n.item()), dtype=torch.uint8)
            dist.recv(blob, src, group=self.group)
            t.copy_(codec.decode_cpu(blob, t.numel(), t.dtype).view(t.shape))

    def broadcast(self, tensors, src: int) -> None:
        me, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        if me == src:
            self.send(tensors, [r for r in range(world) if r != src])
        else:
            self.recv(tensors, src)


_CODEC_DTYPES = (torch.bfloat16, torch.float16, torch.float32) + tuple(
    d for d in (getattr(torch, "float8_e4m3fn", None), getattr(torch, "float8_e5m2", None)) if d is not None)


def _host(state_dict) -> bool:
    ts = list(state_dict.values()) if isinstance(state_dict, dict) else list(state_dict)
    return bool(ts) and all(not t.is_cuda for t in ts)


_ENGINES: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()


def _engine(comm, mode, **kw):
    """One engine per (communicator, mode, options); dropped with the communicator."""
    from .allreduce import get_comm, init

    comm = comm or get_comm() or init()
    per_comm = _ENGINES.setdefault(comm, {})
    key = (mode, tuple(sorted(kw.items())))
    if key not in per_comm:
        per_comm[key] = WeightTransfer(comm, mode=mode, **kw)
    return per_comm[key]


def _progress(items, what: str):
    """tqdm progress over buckets when LZ_PROGRESS=1 (tqdm is optional)."""
    if os.environ.get("LZ_PROGRESS", "0") in ("", "0"):
        return items
    try:
        from tqdm import tqdm
    except ImportError:
        return items
    return tqdm(items, desc=what, unit="bucket")


def _log_bucket(what: str, i: int, bucket) -> None:
    nbytes = sum(t.numel() * t.element_size() for _, t in bucket)
    trace.log.info("[BUCKET] %s %d start tensors=%d bytes=%.1fMB", what, i, len(bucket), nbytes / 2**20)


def send_weights(state_dict, dst, comm=None, mode: str = "split_ans", bucket_bytes: int | None = None,
                 dump_dir: str | None = None, weight_version: int = 0, **kw) -> None:
    """Send a state_dict (name -> tensor) to rank(s) `dst`, bucket by bucket
    (CUDA tensors: native kernels; CPU tensors: :class:`HostTransfer`)."""
    eng = HostTransfer(mode) if _host(state_dict) else _engine(comm, mode, **kw)
    if isinstance(eng, HostTransfer):
        bucket_bytes = bucket_bytes or (512 << 20)
    bb = bucket_bytes or eng.comm.config.update_weight_buffer_bytes
    me = dist.get_rank() if isinstance(eng, HostTransfer) else eng.comm.rank
    trace.log.info("[START] send_weights version=%d mode=%s dst=%s", weight_version, mode, dst)
    nb = 0
    for i, bucket in enumerate(_progress(list(buckets(list(state_dict.items()), bb)), "send_weights")):
        _log_bucket("send", i, bucket)
        if dump_dir:
            dump_tensors(bucket, dump_dir, weight_version, i, group_name=f"src{me}")
        with trace.range(f"send_weights.bucket{i}"):
            eng.send([t for _, t in bucket], dst)
        nb = i + 1
    if dump_dir:
        mark_dump_complete(dump_dir, weight_version, nb)


def recv_weights(state_dict, src: int, comm=None, mode: str = "split_ans", bucket_bytes: int | None = None,
                 **kw) -> dict:
    """Receive into the destination tensors of `state_dict` (same names, shapes, order)."""
    eng = HostTransfer(mode) if _host(state_dict) else _engine(comm, mode, **kw)
    bb = bucket_bytes or (512 << 20 if isinstance(eng, HostTransfer) else eng.comm.config.update_weight_buffer_bytes)
    for i, bucket in enumerate(_progress(list(buckets(list(state_dict.items()), bb)), "recv_weights")):
        _log_bucket("recv", i, bucket)
        with trace.range(f"recv_weights.bucket{i}"):
            eng.recv([t for _, t in bucket], src)
    return state_dict


def broadcast_weights(state_dict, src: int = 0, comm=None, mode: str = "split_ans",
                      bucket_bytes: int | None = None, **kw) -> dict:
    """Every rank calls: `src` sends its state_dict, the others receive into theirs.

    With ``mode="raw"`` and every tensor allocated in the symmetric heap
    (``comm.empty``, same order on all ranks) the update goes zero-copy
    through :meth:`WeightTransfer.broadcast_direct` (relay broadcast for more
    than two ranks): no slots and no receiver copies, in one launch.
    """
    if _host(state_dict):
        eng = HostTransfer(mode)
        for bucket in buckets(list(state_dict.items()), bucket_bytes or (512 << 20)):
            eng.broadcast([t for _, t in bucket], src)
        return state_dict
    eng = _engine(comm, mode, **kw)
    tensors = list(state_dict.values())
    if mode == "raw" and tensors and all(t.is_cuda and eng.comm.is_symmetric(t) for t in tensors):
        trace.log.info("[START] broadcast_weights zero-copy tensors=%d src=%d", len(tensors), src)
        with trace.range("broadcast_weights.direct"):
            eng.broadcast_direct(tensors, src)
        return state_dict
    bb = bucket_bytes or eng.comm.config.update_weight_buffer_bytes
    for i, bucket in enumerate(_progress(list(buckets(list(state_dict.items()), bb)), "broadcast_weights")):
        _log_bucket("broadcast", i, bucket)
        with trace.range(f"broadcast_weights.bucket{i}"):
            eng.broadcast([t for _, t in bucket], src)
    return state_dict


def exchange_metadata(state_dict, src: int, group=None):
    """Receivers learn (name, shape, dtype) of the sender's tensors (host control plane)."""
    meta = [[(k, tuple(v.shape), str(v.dtype)) for k, v in state_dict.items()] if state_dict else None]
    dist.broadcast_object_list(meta, src=src, group=group)
    return meta[0]


def allocate_like(meta, device) -> dict:
    return {k: torch.empty(shape, dtype=getattr(torch, dt.replace("torch.", "")), device=device)
            for k, shape, dt in meta}


# ---------------------------------------------------------------------- dump / manifest
def dump_tensors(named, dump_dir: str, weight_version: int, shard_idx: int, group_name: str = "") -> str:
    """weight_version_XXXXXX/shard_XXXXXX.safetensors + appended manifest.jsonl
    (same layout as back_up/update_weight_from_distributed.py:93-160)."""
    step_dir = os.path.join(dump_dir, f"weight_version_{weight_version:06d}")
    os.makedirs(step_dir, exist_ok=True)
    cpu_state, meta = {}, []
    for name, t in named:
        tt = t.detach().contiguous().cpu()
        cpu_state[name] = tt
        meta.append({"name": name, "dtype": str(tt.dtype).replace("torch.", ""), "shape": list(tt.shape),
                     "numel": tt.numel(), "nbytes": tt.numel() * tt.element_size()})
    base = f"shard_{shard_idx:06d}"
    try:
        from safetensors.torch import save_file

        path = os.path.join(step_dir, base + ".safetensors")
        save_file(cpu_state, path)
        fmt = "safetensors"
    except Exception:
        path = os.path.join(step_dir, base + ".pt")
        torch.save(cpu_state, path)
        fmt = "pt"
    rec = {"time": time.time(), "weight_version": int(weight_version), "group_name": group_name,
           "shard": os.path.basename(path), "num_tensors": len(cpu_state),
           "total_nbytes": int(sum(m["nbytes"] for m in meta)), "tensors": meta, "format": fmt}
    with open(os.path.join(step_dir, "manifest.jsonl"), "a", encoding="utf-8") as f:
        f.write(json.dumps(rec) + "\n")
    return path


COMPLETE_MARKER = "COMPLETE.json"


def mark_dump_complete(dump_dir: str, weight_version: int, num_shards: int) -> str:
    """Record that every shard of a version is written (written last, after
    the final manifest line, through a rename so it appears atomically)."""
    step_dir = os.path.join(dump_dir, f"weight_version_{weight_version:06d}")
    os.makedirs(step_dir, exist_ok=True)
    path = os.path.join(step_dir, COMPLETE_MARKER)
    tmp = path + f".tmp{os.getpid()}"
    with open(tmp, "w", encoding="utf-8") as f:
        json.dump({"weight_version": int(weight_version), "num_shards": int(num_shards), "time": time.time()}, f)
    os.replace(tmp, path)
    return path


def _dump_complete(step_dir: str) -> bool:
    """A version counts only when its marker exists and the manifest lists as
    many distinct shards as the marker promises (a crash part-way through a
    multi-shard dump leaves no marker, or a short manifest)."""
    try:
        with open(os.path.join(step_dir, COMPLETE_MARKER), encoding="utf-8") as f:
            want = int(json.load(f)["num_shards"])
        shards = set()
        with open(os.path.join(step_dir, "manifest.jsonl"), encoding="utf-8") as f:
            for line in f:
                if line.strip():
                    shards.add(json.loads(line)["shard"])
    except (OSError, ValueError, KeyError):
        return False
    return len(shards) >= want and all(os.path.exists(os.path.join(step_dir, s)) for s in shards)


def latest_dump_version(dump_dir: str) -> int | None:
    """Highest weight version under `dump_dir` whose dump completed (None if
    there is none): incomplete versions are skipped, so a resume never picks
    a dump that a crash cut short."""
    if not os.path.isdir(dump_dir):
        return None
    best = None
    for name in os.listdir(dump_dir):
        if not name.startswith("weight_version_"):
            continue
        try:
            v = int(name[len("weight_version_"):])
        except ValueError:
            continue
        if _dump_complete(os.path.join(dump_dir, name)):
            best = v if best is None or v > best else best
    return best


def load_dump(dump_dir: str, weight_version: int) -> dict:
    """Read back every shard of a dumped weight version (bit-exact oracle for receivers)."""
    step_dir = os.path.join(dump_dir, f"weight_version_{weight_version:06d}")
    out = {}
    with open(os.path.join(step_dir, "manifest.jsonl")) as f:
        for line in f:
            rec = json.loads(line)
            p = os.path.join(step_dir, rec["shard"])
            if rec["format"] == "safetensors":
                from safetensors.torch import load_file

                out.update(load_file(p))
            else:
                out.update(torch.load(p))
    return out
