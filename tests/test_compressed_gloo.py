"""Host-orchestrated compressed allreduce variants (CPU oracle codec) on gloo
ranks: results match dist.all_reduce, and streams that exceed the fixed budget
are delivered in full through the overflow message (never truncated)."""
import pytest
import torch

from tests._mp import run_ranks


def _worker(rank, world, variant, n, dtname, ratio, kind):
    import torch
    import torch.distributed as dist

    from results_b200.parallel import compressed

    dtype = getattr(torch, dtname)
    torch.manual_seed(0)
    if kind == "normal":
        xs = [(torch.randn(n) * 1e-2).to(dtype) for _ in range(world)]
    else:  # incompressible bit patterns (finite values)
        xs = [(torch.rand(n) * 2 - 1).to(dtype) for _ in range(world)]
    exact = torch.stack([x.float() for x in xs]).sum(0)
    t = xs[rank].clone()
    compressed.STATS.__init__()
    fn = compressed.VARIANTS[variant]
    if ratio is None:
        fn(t)
    else:
        fn(t, ratio=ratio)
    err = ((t.float() - exact).abs().max() / exact.abs().max()).item()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    return err <= tol, err, compressed.STATS.overflows, compressed.STATS.ratio


@pytest.mark.parametrize("variant,world", [("compressed_twoshot", 2), ("compressed_twoshot", 4),
                                           ("compressed_ring", 2), ("compressed_ring", 4),
                                           ("compressed_nosize", 2)])
@pytest.mark.parametrize("dtname", ["bfloat16", "float32"])
def test_variants_match_allreduce(variant, world, dtname):
    res = run_ranks(_worker, world, backend="gloo", args=(variant, 100_000, dtname, 0.9, "normal"), timeout=300)
    assert all(r[0] for r in res), res


def test_sizeexchange_two_ranks():
    res = run_ranks(_worker, 2, backend="gloo", args=("compressed_sizeexchange", 70_001, "bfloat16", None, "normal"),
                    timeout=300)
    assert all(r[0] for r in res), res


def test_overflow_is_sent_not_truncated():
    # budget ratio 0.3 is far below what bf16 data compresses to (~0.67):
    # every message overflows, and the result must still be exact
    res = run_ranks(_worker, 2, backend="gloo", args=("compressed_twoshot", 200_000, "bfloat16", 0.3, "normal"),
                    timeout=300)
    assert all(r[0] for r in res), res
    assert all(r[2] > 0 for r in res)


def test_incompressible_ring():
    res = run_ranks(_worker, 4, backend="gloo", args=("compressed_ring", 50_000, "float32", 0.65, "uniform"),
                    timeout=300)
    assert all(r[0] for r in res), res


@pytest.mark.parametrize("variant,world,n", [("compressed_twoshot", 3, 10_001), ("compressed_ring", 3, 10_001),
                                             ("compressed_twoshot", 4, 3)])
def test_variants_uneven_sizes(variant, world, n):
    """Element counts that do not divide by the world size, down to fewer
    elements than ranks: chunks of unequal (or zero) length still reduce."""
    res = run_ranks(_worker, world, backend="gloo", args=(variant, n, "float32", 0.9, "normal"), timeout=300)
    assert all(r[0] for r in res), res
