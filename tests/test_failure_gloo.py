"""Failure detection on CPU ranks (gloo): a rank that leaves between steps,
a rank that dies without notice, and a collective whose peer is gone ending
with an error from the short process-group timeout instead of hanging."""
import os
import time

import pytest

from tests._mp import run_ranks

ENV = {"LZ_TEST_PG_TIMEOUT": "6", "LZ_TEST_NO_FINAL_BARRIER": "1"}


def _leave_worker(rank, world, mode):
    import torch
    import torch.distributed as dist

    from results_b200.utils.health import Heartbeat, PeerLost

    hb = Heartbeat(rank, world, period_s=0.1)
    t = torch.ones(16)
    dist.all_reduce(t)  # step 1, everyone present
    dist.barrier()
    if rank == world - 1:
        if mode == "leave":
            hb.leave()
            return "left"
        os._exit(3)  # crash: no notice, heartbeat stops
    deadline = time.time() + 10
    while time.time() < deadline:
        try:
            hb.check(max_age_s=1.0)
        except PeerLost as e:
            return ("detected", e.ranks)
        time.sleep(0.05)
    return ("not detected", [])


@pytest.mark.parametrize("mode", ["leave", "crash"])
def test_survivors_detect_lost_peer(mode):
    res = run_ranks(_leave_worker, 3, backend="gloo", args=(mode,), timeout=120, env=ENV, allow_missing=True)
    for r in (0, 1):
        assert res[r] == ("detected", [2]), res


def _timeout_worker(rank, world):
    import torch
    import torch.distributed as dist

    from results_b200.parallel import sendrecv

    t = torch.ones(1024)
    sendrecv.ring_sendrecv(t)
    if rank == 1:
        return "gone"  # leaves without joining the next collective
    t0 = time.time()
    try:
        sendrecv.ring_sendrecv(t)
    except Exception as e:  # gloo timeout -> error, not a hang
        return ("error", round(time.time() - t0, 1), type(e).__name__)
    return ("no error",)


def test_collective_with_missing_peer_errors():
    res = run_ranks(_timeout_worker, 2, backend="gloo", timeout=120, env=ENV, allow_missing=True)
    assert res[0][0] == "error", res
    assert res[0][1] < 60


def _shrink_worker(rank, world):
    import torch
    import torch.distributed as dist

    from results_b200.parallel import sendrecv
    from results_b200.utils.health import Heartbeat, PeerLost, rebuild_world

    hb = Heartbeat(rank, world, period_s=0.1)
    t = torch.full((1000,), float(rank + 1))
    sendrecv.ring_sendrecv(t)  # step 1 with everyone
    dist.barrier()
    if rank == 2:
        os._exit(5)  # dies between steps without notice
    lost = []
    deadline = time.time() + 10
    while time.time() < deadline and not lost:
        try:
            hb.check(max_age_s=1.0)
            time.sleep(0.05)
        except PeerLost as e:
            lost = e.ranks
    hb.stop()
    new_rank, new_world = rebuild_world(lost, timeout_s=30)
    t = torch.full((1000,), float(rank + 1))
    sendrecv.ring_sendrecv(t)  # step 2 among the survivors
    return lost, new_rank, new_world, float(t[0])


def test_survivors_rebuild_and_continue():
    """Elastic shrink on CPU ranks: rank 2 of 4 dies, the others detect it,
    re-form the group (ranks 0, 1, 3 -> 0, 1, 2) and the next allreduce runs
    on the survivors only."""
    res = run_ranks(_shrink_worker, 4, backend="gloo", timeout=120, env=ENV, allow_missing=True)
    want_sum = 1.0 + 2.0 + 4.0
    got = {r: v for r, v in enumerate(res) if v is not None}
    assert set(got) == {0, 1, 3}, res
    for old, (lost, nr, nw, v) in got.items():
        assert lost == [2] and nw == 3 and nr == [0, 1, 3].index(old) and v == want_sum, res
