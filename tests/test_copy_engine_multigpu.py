"""Copy-engine two-shot (DMA peer reads) and the host-staged PCIe-emulation
path across real GPUs, bit-exact against the fp32 rank-order reference."""
import pytest
import torch

from tests._mp import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world):
    import torch

    from results_b200.config import Config
    from results_b200.parallel.comm import Communicator
    from results_b200.parallel import copy_engine

    comm = Communicator(config=Config(user_bytes=16 << 20, stage_bytes=256 << 20))
    out = []
    for n, pipes in ((1 << 20, 1), (1 << 22, 4), (3 * 8 * 1024, 2)):
        xs = []
        for r in range(world):
            g = torch.Generator(device="cuda").manual_seed(r + n)
            xs.append((torch.randn(n, device="cuda", generator=g) * 1e-2).to(torch.bfloat16))
        acc = xs[0].float().clone()
        for x in xs[1:]:
            acc += x.float()
        ref = acc.to(torch.bfloat16)
        y = torch.empty_like(xs[rank])
        copy_engine.ce_allreduce(xs[rank], y, comm=comm, pipes=pipes)
        torch.cuda.synchronize()
        comm.check()
        out.append(("ce", n, bool(torch.equal(y, ref))))
        t = xs[rank].clone()
        copy_engine.hoststaged_allreduce(t, ctrl=comm.ctrl)
        out.append(("host", n, bool(torch.equal(t, ref))))
    copy_engine.close_host_stages()
    comm.close()
    return out


def test_copy_engine_paths():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_ranks(_worker, 2, backend="nccl", timeout=300)
    bad = [r for rr in res for r in rr if not r[2]]
    assert not bad, bad
