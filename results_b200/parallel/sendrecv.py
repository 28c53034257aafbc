"""Host-orchestrated allreduce algorithms over point-to-point messages.

These are the reference's send/recv algorithms, re-implemented for any
``torch.distributed`` backend (gloo on CPU for the test suite, NCCL on GPUs
as baselines for the native kernels). Each reduces ``t`` in place (sum).

=====================  ======================================================================
algo                   reference
=====================  ======================================================================
naive_twoshot          all-to-all RS + AG, one batch each
                       (single_node_nccl_allreduce_benchmark/naive_sendrecv_allreduce.py:113-172)
hierarchical           intra-node RS -> inter-node AR of the shard -> intra-node AG, with the
                       2-node exchange split in halves (same file :59-96, :174-232)
naive                  flat naive on one node, hierarchical on several; pipelined over two
                       intra-node groups above ``pipeline_min_elements``
                       (16_node_nccl_allreduce_benchmark/naive_sendrecv_allreduce.py:40,226-406)
ring_sendrecv          2(W-1)-step ring, AG receives straight into place
                       (single_node_nccl_allreduce_benchmark/ring_sendrecv_allreduce.py:21-80)
multichannel_ring      K channels (groups) x ring, or halving-doubling per channel for
                       power-of-two W up to ``hd_max_bytes``
                       (16_node_nccl_allreduce_benchmark/ring_sendrecv_allreduce.py:33-313)
rhd_sendrecv           recursive halving-doubling, power-of-two W
                       (single_node_nccl_allreduce_benchmark/recursive_halving_allreduce.py:20-113)
twoshot_collective     reduce_scatter_tensor + all_gather_into_tensor
                       (single_node_nccl_allreduce_benchmark/twoshot_collective_allreduce.py:16-33)
pipelined_twoshot      W=2 only, K=8 sub-chunk exchanges per phase, with a self check
                       (back_up_nccl_allreduce_benchmark/twoshot_allreduce.py:32-168)
naive_alloc            W=2 baseline that allocates per call and rebuilds with torch.cat
                       (back_up_nccl_allreduce_benchmark/naive_sendrecv_allreduce.py:27-76)
=====================  ======================================================================

The compressed send/recv variants live in :mod:`results_b200.parallel.compressed`.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..config import Config

_GROUP_CACHE: dict = {}


def _info(group):
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(ws))
    return rank, ws, ranks


def _exchange(ops):
    if ops:
        for r in dist.batch_isend_irecv(ops):
            r.wait()


def _chunks(t: torch.Tensor, ws: int):
    """W near-equal contiguous chunks (the last one takes the remainder)."""
    n = t.numel()
    base = n // ws
    out = []
    for i in range(ws):
        s = i * base
        e = n if i == ws - 1 else s + base
        out.append(t[s:e])
    return out


# ---------------------------------------------------------------- naive two-shot
def naive_twoshot(t: torch.Tensor, group=None) -> torch.Tensor:
    rank, ws, gr = _info(group)
    if ws == 1:
        return t
    ch = _chunks(t, ws)
    mine = ch[rank]
    recv = [torch.empty_like(mine) for _ in range(ws)]
    ops = []
    for p in range(ws):
        if p == rank:
            continue
        ops.append(dist.P2POp(dist.isend, ch[p].contiguous(), gr[p], group=group))
        ops.append(dist.P2POp(dist.irecv, recv[p], gr[p], group=group))
    _exchange(ops)
    acc = mine.float().clone() if mine.dtype != torch.float32 else mine.clone()
    for p in range(ws):  # rank order
        if p != rank:
            acc += recv[p].float() if recv[p].dtype != torch.float32 else recv[p]
    mine.copy_(acc)
    ops = []
    recv_ag = [torch.empty_like(ch[p]) if p != rank else None for p in range(ws)]
    for p in range(ws):
        if p == rank:
            continue
        ops.append(dist.P2POp(dist.isend, mine.contiguous(), gr[p], group=group))
        ops.append(dist.P2POp(dist.irecv, recv_ag[p], gr[p], group=group))
    _exchange(ops)
    for p in range(ws):
        if p != rank:
            ch[p].copy_(recv_ag[p])
    return t


# ---------------------------------------------------------------- hierarchical
def _node_layout(world: int):
    lws = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    if lws <= 0 or world % lws:
        raise ValueError(f"WORLD_SIZE {world} is not a multiple of LOCAL_WORLD_SIZE {lws}")
    return lws, world // lws


def _hier_groups():
    """(intra_a, intra_b, inter) groups; created collectively on first use."""
    world = dist.get_world_size()
    lws, nn = _node_layout(world)
    key = ("hier", world, lws)
    if key in _GROUP_CACHE:
        return _GROUP_CACHE[key]
    rank = dist.get_rank()
    node, lr = rank // lws, rank % lws
    intra = []
    for _track in range(2):
        mine = None
        for nid in range(nn):
            g = dist.new_group(list(range(nid * lws, (nid + 1) * lws)))
            if nid == node:
                mine = g
        intra.append(mine)
    inter = None
    for l in range(lws):
        g = dist.new_group([nid * lws + l for nid in range(nn)])
        if l == lr:
            inter = g
    _GROUP_CACHE[key] = (intra[0], intra[1], inter)
    return _GROUP_CACHE[key]


def _inter_allreduce(shard: torch.Tensor, inter) -> None:
    ir, iws, igr = _info(inter)
    if iws == 1:
        return
    if iws == 2:
        # two nodes: exchange the shard in two halves in one batch
        peer = igr[1 - ir]
        recv = torch.empty_like(shard)
        h = shard.numel() // 2
        if h == 0:
            ops = [dist.P2POp(dist.isend, shard, peer, group=inter),
                   dist.P2POp(dist.irecv, recv, peer, group=inter)]
        else:
            ops = [dist.P2POp(dist.isend, shard[:h].contiguous(), peer, group=inter),
                   dist.P2POp(dist.irecv, recv[:h], peer, group=inter),
                   dist.P2POp(dist.isend, shard[h:].contiguous(), peer, group=inter),
                   dist.P2POp(dist.irecv, recv[h:], peer, group=inter)]
        _exchange(ops)
        # lower node index first so both nodes add in the same order
        if ir == 0:
            shard.add_(recv)
        else:
            recv.add_(shard)
            shard.copy_(recv)
    else:
        naive_twoshot(shard, inter)


def hierarchical(t: torch.Tensor, group=None, config: Config | None = None) -> torch.Tensor:
    """Intra RS -> inter AR -> intra AG (serial; pipelined halves for large tensors)."""
    cfg = config or Config.from_env()
    world = dist.get_world_size()
    lws, nn = _node_layout(world)
    if nn == 1:
        return naive_twoshot(t, group)
    intra_a, intra_b, inter = _hier_groups()
    if t.numel() >= cfg.pipeline_min_elements and t.numel() >= 2 * lws:
        return _hier_pipelined(t, intra_a, intra_b, inter)
    _hier_serial(t, intra_a, inter)
    return t


def _hier_serial(t, intra, inter):
    rank, ws, gr = _info(intra)
    ch = _chunks(t, ws)
    _rs_only(t, intra)
    _inter_allreduce(ch[rank], inter)
    _ag_only(t, intra)


def _rs_issue(t, group):
    """Post the intra-group reduce-scatter; returns a finalize closure."""
    rank, ws, gr = _info(group)
    ch = _chunks(t, ws)
    recv = [torch.empty_like(ch[rank]) for _ in range(ws)]
    ops = []
    for p in range(ws):
        if p != rank:
            ops.append(dist.P2POp(dist.isend, ch[p].contiguous(), gr[p], group=group))
            ops.append(dist.P2POp(dist.irecv, recv[p], gr[p], group=group))
    works = dist.batch_isend_irecv(ops) if ops else []

    def finalize():
        for w in works:
            w.wait()
        acc = ch[rank].float()
        for p in range(ws):
            if p != rank:
                acc = acc + recv[p].float()
        ch[rank].copy_(acc)
    return finalize


def _ag_issue(t, group):
    rank, ws, gr = _info(group)
    ch = _chunks(t, ws)
    recv = [torch.empty_like(ch[p]) for p in range(ws)]
    ops = []
    for p in range(ws):
        if p != rank:
            ops.append(dist.P2POp(dist.isend, ch[rank].contiguous(), gr[p], group=group))
            ops.append(dist.P2POp(dist.irecv, recv[p], gr[p], group=group))
    works = dist.batch_isend_irecv(ops) if ops else []

    def finalize():
        for w in works:
            w.wait()
        for p in range(ws):
            if p != rank:
                ch[p].copy_(recv[p])
    return finalize


def _inter_issue(shard, inter):
    """Post the 2-node shard exchange (other node counts run it synchronously)."""
    ir, iws, igr = _info(inter)
    if iws != 2:
        _inter_allreduce(shard, inter)
        return lambda: None
    peer = igr[1 - ir]
    recv = torch.empty_like(shard)
    h = shard.numel() // 2
    if h == 0:
        ops = [dist.P2POp(dist.isend, shard.clone(), peer, group=inter),
               dist.P2POp(dist.irecv, recv, peer, group=inter)]
    else:
        ops = [dist.P2POp(dist.isend, shard[:h].clone(), peer, group=inter),
               dist.P2POp(dist.irecv, recv[:h], peer, group=inter),
               dist.P2POp(dist.isend, shard[h:].clone(), peer, group=inter),
               dist.P2POp(dist.irecv, recv[h:], peer, group=inter)]
    works = dist.batch_isend_irecv(ops)

    def finalize():
        for w in works:
            w.wait()
        if ir == 0:
            shard.add_(recv)
        else:
            recv.add_(shard)
            shard.copy_(recv)
    return finalize


def _rs_only(t, group):
    _rs_issue(t, group)()


def _ag_only(t, group):
    _ag_issue(t, group)()


def _hier_pipelined(t, intra_a, intra_b, inter):
    """Halves A and B on independent intra-node groups so the inter-node
    exchange of one half overlaps the intra-node stage of the other:
        t0: RS_A | t1: Ex_A || RS_B | t2: AG_A || Ex_B | t3: AG_B
    """
    h = t.numel() // 2
    A, B = t[:h], t[h:]
    ra, wa, _ = _info(intra_a)
    rb, wb, _ = _info(intra_b)
    _rs_issue(A, intra_a)()
    fin_ex_a = _inter_issue(_chunks(A, wa)[ra], inter)
    fin_rs_b = _rs_issue(B, intra_b)
    fin_ex_a()
    fin_rs_b()
    fin_ag_a = _ag_issue(A, intra_a)
    fin_ex_b = _inter_issue(_chunks(B, wb)[rb], inter)
    fin_ag_a()
    fin_ex_b()
    _ag_issue(B, intra_b)()
    return t


# ---------------------------------------------------------------- ring
def ring_sendrecv(t: torch.Tensor, group=None) -> torch.Tensor:
    rank, ws, gr = _info(group)
    if ws == 1:
        return t
    ch = _chunks(t, ws)
    right, left = gr[(rank + 1) % ws], gr[(rank - 1) % ws]
    buf = torch.empty(max(c.numel() for c in ch), dtype=t.dtype, device=t.device)
    si, ri = rank, (rank - 1) % ws
    for _ in range(ws - 1):  # reduce-scatter
        rb = buf[: ch[ri].numel()]
        _exchange([dist.P2POp(dist.isend, ch[si].contiguous(), right, group=group),
                   dist.P2POp(dist.irecv, rb, left, group=group)])
        ch[ri].add_(rb)
        si, ri = ri, (ri - 1) % ws
    si, ri = (rank + 1) % ws, rank
    for _ in range(ws - 1):  # all-gather, received straight into place
        _exchange([dist.P2POp(dist.isend, ch[si].contiguous(), right, group=group),
                   dist.P2POp(dist.irecv, ch[ri], left, group=group)])
        si, ri = ri, (ri - 1) % ws
    return t


# ---------------------------------------------------------------- recursive halving-doubling
def rhd_sendrecv(t: torch.Tensor, group=None) -> torch.Tensor:
    rank, ws, gr = _info(group)
    if ws == 1:
        return t
    if ws & (ws - 1):
        raise ValueError("recursive halving-doubling needs a power-of-two world size")
    lo, hi = 0, t.numel()
    steps = []
    dist_ = ws // 2
    while dist_ >= 1:  # halving
        peer = rank ^ dist_
        mid = lo + (hi - lo) // 2
        if rank & dist_:
            keep, send = (mid, hi), (lo, mid)
        else:
            keep, send = (lo, mid), (mid, hi)
        recv = torch.empty(keep[1] - keep[0], dtype=t.dtype, device=t.device)
        _exchange([dist.P2POp(dist.isend, t[send[0]:send[1]].contiguous(), gr[peer], group=group),
                   dist.P2POp(dist.irecv, recv, gr[peer], group=group)])
        t[keep[0]:keep[1]].add_(recv)
        steps.append((peer, keep, send))
        lo, hi = keep
        dist_ //= 2
    for peer, keep, send in reversed(steps):  # doubling
        _exchange([dist.P2POp(dist.isend, t[keep[0]:keep[1]].contiguous(), gr[peer], group=group),
                   dist.P2POp(dist.irecv, t[send[0]:send[1]], gr[peer], group=group)])
    return t


# ---------------------------------------------------------------- multi-channel
def _channel_groups(k: int):
    key = ("chan", dist.get_world_size(), k)
    if key not in _GROUP_CACHE:
        _GROUP_CACHE[key] = [dist.new_group(list(range(dist.get_world_size()))) for _ in range(k)]
    return _GROUP_CACHE[key]


def multichannel_ring(t: torch.Tensor, group=None, config: Config | None = None) -> torch.Tensor:
    """K independent communicators each reduce 1/K of the tensor (ring or
    halving-doubling by size), concurrently (CUDA: one stream per channel)."""
    cfg = config or Config.from_env()
    ws = dist.get_world_size(group)
    nbytes = t.numel() * t.element_size()
    use_hd = (ws & (ws - 1)) == 0 and nbytes <= cfg.hd_max_bytes
    if use_hd:
        k = 1 if nbytes <= (8 << 20) else (2 if nbytes <= (32 << 20) else 4)
    else:
        k = 1 if nbytes < (32 << 20) else (2 if nbytes < (128 << 20) else 4)
    k = max(1, min(k, cfg.ring_channels))
    groups = _channel_groups(cfg.ring_channels)[:k]
    parts = _chunks(t, k)
    fn = rhd_sendrecv if use_hd else ring_sendrecv
    if t.is_cuda:
        cur = torch.cuda.current_stream()
        streams = [torch.cuda.Stream() for _ in range(k)]
        for s, p, g in zip(streams, parts, groups):
            s.wait_stream(cur)
            with torch.cuda.stream(s):
                fn(p, g)
        for s in streams:
            cur.wait_stream(s)
    else:
        import threading

        errs = []

        def run(p, g):
            try:
                fn(p, g)
            except BaseException as e:  # pragma: no cover - surfaced below
                errs.append(e)

        ths = [threading.Thread(target=run, args=(p, g)) for p, g in zip(parts, groups)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        if errs:
            raise errs[0]
    return t


# ---------------------------------------------------------------- collective two-shot
def twoshot_collective(t: torch.Tensor, group=None) -> torch.Tensor:
    rank, ws, _ = _info(group)
    if ws == 1:
        return t
    n = t.numel()
    pad = (-n) % ws
    flat = torch.cat([t, t.new_zeros(pad)]) if pad else t
    shard = torch.empty(flat.numel() // ws, dtype=t.dtype, device=t.device)
    dist.reduce_scatter_tensor(shard, flat, group=group)
    dist.all_gather_into_tensor(flat, shard, group=group)
    if pad:
        t.copy_(flat[:n])
    return t


# ---------------------------------------------------------------- W=2 variants
def pipelined_twoshot(t: torch.Tensor, group=None, k: int = 8) -> torch.Tensor:
    """Two ranks: K sequential sub-chunk exchanges for RS, then K for AG."""
    rank, ws, gr = _info(group)
    if ws != 2:
        raise ValueError("pipelined_twoshot is a two-rank algorithm")
    peer = gr[1 - rank]
    ch = _chunks(t, 2)
    mine, other = ch[rank], ch[1 - rank]
    subs_o, subs_m = _chunks(other, k), _chunks(mine, k)
    for so, sm in zip(subs_o, subs_m):
        r = torch.empty_like(sm)
        _exchange([dist.P2POp(dist.isend, so.contiguous(), peer, group=group),
                   dist.P2POp(dist.irecv, r, peer, group=group)])
        if rank == 0:
            sm.add_(r)
        else:
            r.add_(sm)
            sm.copy_(r)
    for so, sm in zip(subs_o, subs_m):
        _exchange([dist.P2POp(dist.isend, sm.contiguous(), peer, group=group),
                   dist.P2POp(dist.irecv, so, peer, group=group)])
    return t


def naive_alloc(t: torch.Tensor, group=None) -> torch.Tensor:
    """Two-rank baseline without buffer reuse: allocates per call, rebuilds with cat."""
    rank, ws, gr = _info(group)
    if ws != 2:
        raise ValueError("naive_alloc is a two-rank algorithm")
    peer = gr[1 - rank]
    half = t.numel() // 2
    parts = [t[:half].clone(), t[half:].clone()]
    recv = torch.empty_like(parts[rank])
    _exchange([dist.P2POp(dist.isend, parts[1 - rank], peer, group=group),
               dist.P2POp(dist.irecv, recv, peer, group=group)])
    red = parts[rank] + recv if rank == 0 else recv + parts[rank]
    other = torch.empty_like(parts[1 - rank])
    _exchange([dist.P2POp(dist.isend, red, peer, group=group),
               dist.P2POp(dist.irecv, other, peer, group=group)])
    full = torch.cat([red, other]) if rank == 0 else torch.cat([other, red])
    t.copy_(full)
    return t


def verify_correctness(fn, group=None, sizes=(1024, 1 << 20, 16 << 20), device=None) -> bool:
    """Fill rank+1, allreduce, expect sum(1..W) everywhere
    (back_up_nccl_allreduce_benchmark/twoshot_allreduce.py:156-168)."""
    rank, ws, _ = _info(group)
    expect = ws * (ws + 1) / 2
    for n in sizes:
        x = torch.full((n,), float(rank + 1), device=device)
        fn(x, group)
        if not torch.all(x == expect):
            return False
    return True


ALGOS = {
    "naive_twoshot": naive_twoshot,
    "naive": lambda t, group=None: hierarchical(t, group),
    "hierarchical": hierarchical,
    "ring_sendrecv": ring_sendrecv,
    "rhd_sendrecv": rhd_sendrecv,
    "multichannel_ring": multichannel_ring,
    "twoshot_collective": twoshot_collective,
    "pipelined_twoshot": pipelined_twoshot,
    "naive_alloc": naive_alloc,
}


def allreduce(t: torch.Tensor, algo: str, group=None) -> torch.Tensor:
    try:
        fn = ALGOS[algo]
    except KeyError:
        raise ValueError(f"unknown send/recv allreduce {algo!r}") from None
    return fn(t, group=group)
