"""DDP communication hook on CPU (gloo) ranks: gradients after backward equal
those of stock DDP (mean over ranks), for the plain and the compressed hook."""
import pytest

from tests._mp import run_ranks


def _worker(rank, world, compressed):
    import torch
    import torch.distributed as dist

    from results_b200.parallel import ddp

    def make():
        torch.manual_seed(0)
        return torch.nn.Sequential(torch.nn.Linear(64, 128), torch.nn.GELU(), torch.nn.Linear(128, 17))

    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(32, 64, generator=g)
    ref_model = torch.nn.parallel.DistributedDataParallel(make())
    ref_model(x).square().mean().backward()
    ours = torch.nn.parallel.DistributedDataParallel(make(), bucket_cap_mb=0.01)
    state = ddp.register(ours, compressed=compressed)
    ours(x).square().mean().backward()
    dist.barrier()
    diffs = [float((a.grad - b.grad).abs().max()) for a, b in zip(ours.parameters(), ref_model.parameters())]
    return max(diffs), state.calls


@pytest.mark.parametrize("compressed", [False, True])
def test_ddp_hook_matches_stock_ddp(compressed):
    res = run_ranks(_worker, 2, args=(compressed,))
    for err, calls in res:
        assert calls >= 1
        assert err <= 1e-6, res
