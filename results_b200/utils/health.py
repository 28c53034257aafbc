"""Failure detection on the host: heartbeats and explicit leave notices in
the torch.distributed store, checked before a collective is launched.

A rank that stops (crash, exit, hang) stops refreshing ``lz/hb/<rank>``;
a rank that leaves on purpose writes ``lz/left/<rank>``. ``check`` raises
:class:`PeerLost` naming the missing ranks, so survivors never launch a
kernel that would wait on a dead peer. Device-side waits are additionally
bounded (``Config.timeout_s``) and report through the status word
(:meth:`Communicator.check`).

The reference has no failure detection (torchrun only reports the child
failure, raw/a.txt:585-604 of the reference); this is new.
"""
from __future__ import annotations

import threading
import time

import torch.distributed as dist


class PeerLost(RuntimeError):
    """One or more peers stopped heart-beating or announced that they left."""

    def __init__(self, ranks, reason):
        super().__init__(f"peers {sorted(ranks)} lost: {reason}")
        self.ranks = sorted(ranks)


def _store():
    from torch.distributed.distributed_c10d import _get_default_store

    return _get_default_store()


class Heartbeat:
    """Background thread publishing this rank's liveness every `period_s`."""

    def __init__(self, rank: int, world: int, period_s: float = 0.2, store=None, prefix: str = "lz"):
        self.rank, self.world, self.period_s = rank, world, period_s
        self.store = store or _store()
        self.prefix = prefix
        self._stop = threading.Event()
        self._beat()
        self._th = threading.Thread(target=self._run, daemon=True)
        self._th.start()

    def _beat(self):
        self.store.set(f"{self.prefix}/hb/{self.rank}", repr(time.time()))

    def _run(self):
        while not self._stop.wait(self.period_s):
            try:
                self._beat()
            except Exception:
                return

    def leave(self):
        """Announce a clean departure (call between steps, nothing in flight)."""
        self._stop.set()
        self._th.join()
        self.store.set(f"{self.prefix}/left/{self.rank}", "1")

    def stop(self):
        self._stop.set()
        self._th.join()

    def check(self, max_age_s: float = 2.0) -> None:
        """Raise PeerLost if a peer left or has not beaten for `max_age_s`."""
        now = time.time()
        lost, left = [], []
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.store.check([f"{self.prefix}/left/{r}"]):
                left.append(r)
                continue
            try:
                ts = float(self.store.get(f"{self.prefix}/hb/{r}").decode())
            except Exception:
                lost.append(r)
                continue
            if now - ts > max_age_s:
                lost.append(r)
        if left or lost:
            reason = []
            if left:
                reason.append(f"left {left}")
            if lost:
                reason.append(f"no heartbeat for > {max_age_s}s {lost}")
            raise PeerLost(left + lost, "; ".join(reason))


def wait_for_peers(hb: Heartbeat, timeout_s: float = 10.0) -> None:
    deadline = time.time() + timeout_s
    while True:
        try:
            hb.check(max_age_s=timeout_s)
            return
        except PeerLost:
            if time.time() > deadline:
                raise
            time.sleep(0.05)


_GENERATION = [0]


def rebuild_world(lost, timeout_s: float = 60.0, backend: str | None = None) -> tuple[int, int]:
    """Elastic shrink: the surviving ranks re-form the default process group
    without the `lost` ranks and return their (new rank, new world size).

    Every survivor calls it (between steps, with nothing in flight) after a
    :class:`PeerLost`. The default group is torn down locally, then
    re-initialised over the same rendezvous store under a per-generation
    prefix, so stale keys of the old group never mix with the new one. Ranks
    keep their order. The store must outlive the lost ranks (torchrun's agent
    store does; with a rank-hosted store, rank 0 must survive). Native
    communicators of the old group are abandoned by the caller
    (``Communicator.abandon``) and created anew on the new group.
    """
    store = _store()
    old_rank, old_world = dist.get_rank(), dist.get_world_size()
    backend = backend or dist.get_backend()
    survivors = [r for r in range(old_world) if r not in set(lost)]
    if old_rank not in survivors:
        raise ValueError(f"rank {old_rank} is listed as lost")
    _GENERATION[0] += 1
    gen = _GENERATION[0]
    try:
        dist.destroy_process_group()
    except Exception:
        pass
    import datetime

    new_rank, new_world = survivors.index(old_rank), len(survivors)
    prefix = dist.PrefixStore(f"lz/gen{gen}/", store)
    dist.init_process_group(backend=backend, store=prefix, rank=new_rank, world_size=new_world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return new_rank, new_world

