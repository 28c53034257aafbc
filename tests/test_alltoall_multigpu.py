"""All-to-all across real GPUs (one process per GPU): raw into a plain
output, raw zero-copy into a symmetric output, and split+rANS compressed,
each checked bit for bit against the chunks every rank generated."""
import pytest
import torch

from tests._mp import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world):
    import torch

    from results_b200.config import Config
    from results_b200.parallel.alltoall import all_to_all
    from results_b200.parallel.comm import Communicator

    comm = Communicator(config=Config(user_bytes=128 << 20, stage_bytes=128 << 20, timeout_s=10.0))
    out = []
    for mode in ("raw", "raw_symmetric", "compressed"):
        for dtype in (torch.bfloat16, torch.float32):
            chunk = 70000 + 8 * world
            xs = []
            for r in range(world):
                g = torch.Generator(device="cuda").manual_seed(1000 + r)
                xs.append((torch.randn(chunk * world, device="cuda", generator=g) * 0.02).to(dtype))
            ref = torch.cat([xs[src].view(world, chunk)[rank] for src in range(world)])
            if mode == "raw_symmetric":
                comm.reset_alloc()
                res = comm.empty(chunk * world, dtype)
            else:
                res = torch.empty_like(xs[rank])
            for _ in range(3):
                all_to_all(xs[rank], res, compress=(mode == "compressed"), comm=comm)
            torch.cuda.synchronize()
            comm.check()
            ok = torch.equal(res.view(torch.uint8), ref.view(torch.uint8))
            out.append((mode, str(dtype), "ok" if ok else "MISMATCH"))
    comm.close()
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_all_to_all(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = run_ranks(_worker, world, backend="nccl", timeout=600, env={"NCCL_DEBUG": "WARN"})
    bad = [r for rank_res in res for r in rank_res if r[-1] != "ok"]
    assert not bad, bad
