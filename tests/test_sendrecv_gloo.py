"""Send/recv reference algorithms on gloo CPU ranks, checked against
torch.distributed.all_reduce (the CPU/gloo configuration: fp32 and bf16 at 1 KB, 1 MB
and 64 MB, values N(0,1) from torch.manual_seed(0))."""
import pytest
import torch

from tests._mp import run_ranks

SIZES = {"1KB": 1 << 10, "1MB": 1 << 20, "64MB": 64 << 20}


def _worker(rank, world, algos, sizes, dtypes, env_lws):
    import os

    import torch
    import torch.distributed as dist

    from results_b200.parallel import sendrecv

    if env_lws:
        os.environ["LOCAL_WORLD_SIZE"] = str(env_lws)
    out = []
    for dtname in dtypes:
        dtype = getattr(torch, dtname)
        es = torch.empty((), dtype=dtype).element_size()
        for label in sizes:
            n = SIZES[label] // es
            torch.manual_seed(0)
            xs = [torch.randn(n) for _ in range(world)]
            ref = xs[rank].to(dtype).clone()
            dist.all_reduce(ref)
            exact = torch.stack([x.to(dtype).float() for x in xs]).sum(0)
            for algo in algos:
                if algo == "rhd_sendrecv" and world & (world - 1):
                    continue
                if algo in ("pipelined_twoshot", "naive_alloc") and world != 2:
                    continue
                t = xs[rank].to(dtype).clone()
                sendrecv.allreduce(t, algo)
                tol = 1e-4 if dtype == torch.float32 else 2.5e-2
                err = ((t.float() - exact).abs().max() / exact.abs().max()).item()
                err_nccl = ((t.float() - ref.float()).abs().max() / exact.abs().max()).item()
                out.append((algo, dtname, label, err <= tol and err_nccl <= 2 * tol, err))
    return out


ALGOS = ["naive_twoshot", "ring_sendrecv", "rhd_sendrecv", "twoshot_collective", "multichannel_ring",
         "pipelined_twoshot", "naive_alloc", "hierarchical"]


@pytest.mark.parametrize("world", [2, 4])
def test_algorithms_small(world):
    res = run_ranks(_worker, world, backend="gloo",
                    args=(ALGOS, ["1KB", "1MB"], ["float32", "bfloat16"], None), timeout=300)
    bad = [r for rr in res for r in rr if not r[3]]
    assert not bad, bad
    assert len(res[0]) > 0


def test_algorithms_64mb_world2():
    """The CPU/gloo configuration at the 64 MB size: ring, two-shot and RHD."""
    res = run_ranks(_worker, 2, backend="gloo",
                    args=(["ring_sendrecv", "naive_twoshot", "rhd_sendrecv", "twoshot_collective"],
                          ["64MB"], ["float32", "bfloat16"], None), timeout=600)
    bad = [r for rr in res for r in rr if not r[3]]
    assert not bad, bad


def test_hierarchical_two_fake_nodes():
    """4 ranks as 2 'nodes' of 2 (LOCAL_WORLD_SIZE=2): serial and pipelined paths."""
    res = run_ranks(_worker, 4, backend="gloo",
                    args=(["hierarchical"], ["1KB", "64MB"], ["float32"], 2), timeout=600,
                    env={"LZ_PIPELINE_MIN_ELEMENTS": str(1 << 20)})
    bad = [r for rr in res for r in rr if not r[3]]
    assert not bad, bad


def _verify_worker(rank, world):
    from results_b200.parallel import sendrecv

    return all(sendrecv.verify_correctness(sendrecv.ALGOS[a], sizes=(1024, 1 << 16))
               for a in ("naive_twoshot", "ring_sendrecv", "rhd_sendrecv", "pipelined_twoshot"))


def test_verify_correctness_rank_fill():
    assert all(run_ranks(_verify_worker, 2, backend="gloo", timeout=120))


def test_world8_ring_and_rhd():
    res = run_ranks(_worker, 8, backend="gloo",
                    args=(["ring_sendrecv", "rhd_sendrecv", "naive_twoshot"], ["1KB", "1MB"], ["float32"], None),
                    timeout=300)
    bad = [r for rr in res for r in rr if not r[3]]
    assert not bad, bad


def _pattern_worker(rank, world, nbytes, rounds):
    import torch
    import torch.distributed as dist

    wrong = 0
    for it in range(rounds):
        if rank == 0:
            buf = (torch.arange(nbytes, dtype=torch.int64) * 7 + it).remainder(251).to(torch.uint8)
            reqs = [dist.isend(buf, dst=d) for d in range(1, world)]
            for r in reqs:
                r.wait()
        else:
            buf = torch.zeros(nbytes, dtype=torch.uint8)
            dist.irecv(buf, src=0).wait()
            want = (torch.arange(nbytes, dtype=torch.int64) * 7 + it).remainder(251).to(torch.uint8)
            wrong += int((buf != want).sum().item())
    return wrong


@pytest.mark.parametrize("world", [2, 3])
def test_isend_irecv_fill_pattern_consistency(world):
    """Point-to-point consistency (the reference's isend/irecv byte-pattern
    test): rank 0 sends a position-dependent uint8 pattern to every other
    rank, which counts wrong bytes; repeated rounds change the pattern."""
    res = run_ranks(_pattern_worker, world, args=(3 << 20, 3))
    assert res == [0] * world, res


def _odd_worker(rank, world, n):
    import torch
    import torch.distributed as dist

    from results_b200.parallel import sendrecv

    torch.manual_seed(0)
    xs = [torch.randn(n) for _ in range(world)]
    exact = torch.stack(xs).sum(0)
    out = []
    for algo in ("naive_twoshot", "ring_sendrecv", "twoshot_collective", "multichannel_ring"):
        t = xs[rank].clone()
        sendrecv.allreduce(t, algo)
        out.append((algo, float((t - exact).abs().max())))
    if world & (world - 1) == 0:
        t = xs[rank].clone()
        sendrecv.allreduce(t, "rhd_sendrecv")
        out.append(("rhd_sendrecv", float((t - exact).abs().max())))
    return out


@pytest.mark.parametrize("world,n", [(3, 1001), (4, 7), (2, 1)])
def test_algorithms_uneven_sizes(world, n):
    """Element counts that do not divide by the world size (and smaller than
    it): every send/recv algorithm still sums exactly (fp32, tolerance of the
    summation order)."""
    res = run_ranks(_odd_worker, world, backend="gloo", args=(n,), timeout=300)
    bad = [r for rr in res for r in rr if not r[1] <= 1e-5]
    assert not bad, bad
