"""All-to-all on CPU (gloo) ranks: raw and LZC1-compressed exchanges must
equal dist.all_to_all_single of the raw chunks bit for bit."""
import pytest

from tests._mp import run_ranks


def _worker(rank, world, dtname, n):
    import torch
    import torch.distributed as dist

    from results_b200.parallel.alltoall import all_to_all

    dtype = getattr(torch, dtname)
    g = torch.Generator().manual_seed(40 + rank)
    x = (torch.randn(n * world, generator=g) * 0.02).to(dtype)
    ref = torch.empty_like(x)
    dist.all_to_all_single(ref, x)
    raw = all_to_all(x)
    cz = all_to_all(x, compress=True)
    es = 2 if dtype != torch.float32 else 4
    return (torch.equal(raw.view(torch.uint8), ref.view(torch.uint8)),
            torch.equal(cz.view(torch.uint8), ref.view(torch.uint8)), es)


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("dtname", ["bfloat16", "float32"])
def test_all_to_all_cpu_raw_and_compressed(world, dtname):
    res = run_ranks(_worker, world, args=(dtname, 70001))
    assert all(r[0] and r[1] for r in res), res
