"""Device-side failure path on one GPU: a kernel waiting on a flag that
nothing sets gives up after its bound, reports LZ_ERR_TIMEOUT through the
host-mapped status word, and the CUDA context stays usable."""
import datetime
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    import torch.distributed as dist

    from results_b200._native import CollectiveTimeout
    from results_b200.config import Config
    from results_b200.parallel.comm import Communicator
    from tests._mp import free_port

    created = False
    if not dist.is_initialized():
        store = dist.TCPStore("127.0.0.1", free_port(), 1, True, timeout=datetime.timedelta(seconds=30))
        dist.init_process_group("gloo", store=store, rank=0, world_size=1)
        created = True
    comm = Communicator(config=Config(user_bytes=16 << 20, stage_bytes=16 << 20, oneshot_bytes=1 << 20))
    try:
        comm.test_wait_timeout(0.2)
        torch.cuda.synchronize()
        st = comm.status()
        assert st & 0xFF == 1, hex(st)  # LZ_ERR_TIMEOUT
        assert (st >> 8) & 0xFF == 9  # phase of the test hook
        with pytest.raises(CollectiveTimeout):
            comm.check()
        comm.clear_status()
        assert comm.status() == 0
        x = torch.randn(1 << 20, device="cuda")
        y = (x * 2).sum()
        torch.cuda.synchronize()
        assert torch.isfinite(y)
    finally:
        comm.abandon()
        if created:
            dist.destroy_process_group()
