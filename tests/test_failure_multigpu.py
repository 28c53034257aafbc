"""A rank leaves a 2-GPU job between steps (no kernels in flight). The
survivor learns it on the host from the store before its next launch and
raises PeerLost instead of launching a kernel that would wait on the gone
peer. NVLS is off (NCCL_NVLS_ENABLE=0, no multicast object) and the kernels
use plain peer loads/stores."""
import pytest
import torch

from tests._mp import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world):
    import time

    import torch

    from results_b200.config import Config
    from results_b200.parallel.comm import Communicator
    from results_b200.utils.health import PeerLost

    comm = Communicator(config=Config(user_bytes=16 << 20, stage_bytes=64 << 20, use_multicast=False,
                                      timeout_s=2.0))
    hb = comm.attach_heartbeat(period_s=0.1)
    x = torch.ones(1 << 16, device="cuda")
    for _ in range(2):
        comm.guard()
        comm.allreduce_(x, algo="twoshot")
    torch.cuda.synchronize()
    comm.check()
    ok_sum = float(x[0].item())
    comm.barrier_host()
    if rank == 1:
        hb.leave()          # between steps: nothing of ours is in flight
        comm.abandon()
        return ("left", ok_sum)
    deadline = time.time() + 10
    while time.time() < deadline:
        try:
            comm.guard(max_age_s=1.0)
        except PeerLost as e:
            comm.abandon()
            return ("detected", e.ranks, ok_sum)
        time.sleep(0.05)
    comm.abandon()
    return ("not detected",)


def test_peer_leaves_between_steps():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_ranks(_worker, 2, backend="nccl", timeout=180,
                    env={"NCCL_NVLS_ENABLE": "0", "LZ_TEST_PG_TIMEOUT": "20", "LZ_TEST_NO_FINAL_BARRIER": "1"},
                    allow_missing=True)
    assert res[0][0] == "detected" and res[0][1] == [1], res
    assert res[0][2] == 4.0 and res[1] == ("left", 4.0)
