"""Copy-engine two-shot (DMA transfers, SM accumulation) and the host-staged
PCIe-emulation path across real GPUs, bit-exact against the fp32 rank-order
reference. Covers the staged path (ordinary tensors) and the zero-copy
pipelined path (symmetric input and output), several chunk counts, three
dtypes and back-to-back calls (the call counter and flags carry over)."""
import pytest
import torch

from tests._mp import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _inputs(world, n, dtype, seed):
    xs = []
    for r in range(world):
        g = torch.Generator(device="cuda").manual_seed(r + seed)
        xs.append((torch.randn(n, device="cuda", generator=g) * 1e-2).to(dtype))
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()
    return xs, acc.to(dtype)


def _worker(rank, world):
    import torch

    from results_b200.config import Config
    from results_b200.parallel.comm import Communicator
    from results_b200.parallel import copy_engine

    comm = Communicator(config=Config(user_bytes=256 << 20, stage_bytes=256 << 20))
    out = []
    for n, pipes in ((1 << 20, 1), (1 << 22, 4), (3 * 8 * 1024, 2), (1 << 20, 100)):
        xs, ref = _inputs(world, n, torch.bfloat16, n)
        y = torch.empty_like(xs[rank])
        copy_engine.ce_allreduce(xs[rank], y, comm=comm, pipes=pipes)
        torch.cuda.synchronize()
        comm.check()
        out.append(("ce_staged", n, pipes, bool(torch.equal(y, ref))))
        t = xs[rank].clone()
        copy_engine.hoststaged_allreduce(t, ctrl=comm.ctrl)
        out.append(("host", n, bool(torch.equal(t, ref))))
    # zero-copy pipelined path: symmetric, distinct input and output
    x = comm.empty(1 << 24, torch.bfloat16)
    y = comm.empty(1 << 24, torch.bfloat16)
    for dtype, n, pipes in ((torch.bfloat16, 1 << 24, 0), (torch.bfloat16, 1 << 24, 7), (torch.float16, 1 << 22, 3),
                            (torch.float32, 1 << 22, 0), (torch.bfloat16, 16 * world, 1),
                            (torch.bfloat16, 5 * 8 * world * 1000, 64)):
        xs, ref = _inputs(world, n, dtype, 7 * n + 1)
        xv = x.view(torch.uint8)[: n * xs[0].element_size()].view(dtype)
        yv = y.view(torch.uint8)[: n * xs[0].element_size()].view(dtype)
        assert copy_engine.is_zero_copy(comm, xv, yv)
        xv.copy_(xs[rank])
        for rep in range(2):
            yv.fill_(-1)
            copy_engine.ce_allreduce(xv, yv, comm=comm, pipes=pipes)
            torch.cuda.synchronize()
            comm.check()
            out.append(("ce_zero_copy", str(dtype), n, pipes, rep, bool(torch.equal(yv, ref))))
    copy_engine.close_host_stages()
    comm.close()
    return out


def test_copy_engine_paths():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_ranks(_worker, 2, backend="nccl", timeout=300)
    bad = [r for rr in res for r in rr if not r[-1]]
    assert not bad, bad


def test_copy_engine_paths_4():
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    res = run_ranks(_worker, 4, backend="nccl", timeout=300)
    bad = [r for rr in res for r in rr if not r[-1]]
    assert not bad, bad
