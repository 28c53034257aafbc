"""Native allreduce across real GPUs (one process per GPU, NVLink peer memory and
NVLS). Runs with every available GPU count among 2, 4, 8."""
import pytest
import torch

from tests._mp import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _inputs(world, n, dtype, seed):
    xs = []
    for r in range(world):
        g = torch.Generator(device="cuda").manual_seed(seed * 100 + r)
        xs.append((torch.randn(n, device="cuda", generator=g) * 1e-2).to(dtype))
    return xs


def _ordered(t):
    """Float bit patterns as integers whose differences count ulps."""
    if t.element_size() == 2:
        u = t.view(torch.int16).to(torch.int32)
        return torch.where(u < 0, -(u & 0x7FFF), u)
    u = t.view(torch.int32).to(torch.int64)
    return torch.where(u < 0, -(u & 0x7FFFFFFF), u)


def _worker(rank, world, cases):
    import torch

    from results_b200.config import Config
    from results_b200.parallel.comm import Communicator

    cfg = Config(user_bytes=256 << 20, stage_bytes=256 << 20, oneshot_bytes=4 << 20, timeout_s=10.0)
    comm = Communicator(config=cfg)
    out = []
    for (algo, dtname, n, sym, exact) in cases:
        dtype = getattr(torch, dtname)
        if algo.startswith("nvls") and not comm.has_multicast:
            out.append((algo, dtname, n, sym, "skipped-no-multicast"))
            continue
        xs = _inputs(world, n, dtype, seed=n % 9973)
        ref_acc = xs[0].float().clone()
        for x in xs[1:]:
            ref_acc += x.float()
        ref = ref_acc.to(dtype)
        if algo.startswith("compressed"):
            from results_b200.parallel.compressed import compressed_allreduce

            res = torch.empty_like(xs[rank])
            for _ in range(3):
                compressed_allreduce(xs[rank], res, comm=comm, multicast=algo.endswith("_mc"),
                                     hybrid="hybrid" in algo)
        elif algo == "ce_sym":  # zero-copy copy-engine path: symmetric, distinct buffers
            comm.reset_alloc()
            xin, res = comm.empty(n, dtype), comm.empty(n, dtype)
            xin.copy_(xs[rank])
            for _ in range(3):
                res.fill_(0)
                comm.allreduce_(xin, res, algo="ce")
            res = res.clone()
        elif sym:
            comm.reset_alloc()
            buf = comm.empty(n, dtype)
            for _ in range(3):
                buf.copy_(xs[rank])
                comm.allreduce_(buf, algo=algo)
            res = buf.clone()
        else:
            res = torch.empty_like(xs[rank])
            for _ in range(3):
                comm.allreduce_(xs[rank], res, algo=algo)
        torch.cuda.synchronize()
        comm.check()
        if exact == "ulp1" and dtype == torch.float32:
            # NVLS adds fp32 inputs inside the switch in its own order: both it and the
            # rank-order reference lie within (W-1) u sum|x| of the exact sum (u = 2^-24),
            # so they may differ by many ulps of a near-cancelling result; check that bound
            exact_sum = torch.zeros(n, dtype=torch.float64, device="cuda")
            abs_sum = torch.zeros_like(exact_sum)
            for x in xs:
                exact_sum += x.double()
                abs_sum += x.double().abs()
            bound = (world - 1) * 2.0 ** -24 * abs_sum * 1.0001 + 1e-45
            excess = ((res.double() - exact_sum).abs() - bound).max().item()
            err = excess
            ok = excess <= 0
        elif exact == "ulp1":  # 16-bit NVLS: fp32 in the switch, rounded once: within 1 ulp
            err = int((_ordered(res) - _ordered(ref)).abs().max().item())
            ok = err <= 1
        elif exact:
            ok = torch.equal(res, ref)
            err = (res.float() - ref.float()).abs().max().item()
        else:
            err = ((res.float() - ref_acc).abs().max() / ref_acc.abs().max().clamp_min(1e-30)).item()
            ok = err < {torch.float32: 1e-5, torch.float16: 5e-3, torch.bfloat16: 2e-2}[dtype]
        out.append((algo, dtname, n, sym, "ok" if ok else f"MISMATCH err={err}"))
    comm.close()
    return out


CASES = [
    ("oneshot", "bfloat16", 1000, False, True),
    ("oneshot", "float32", 1 << 16, False, True),
    ("twoshot", "bfloat16", (1 << 20) + 64, False, True),
    ("twoshot", "float16", 1 << 20, False, True),
    ("twoshot", "bfloat16", 1 << 21, True, True),
    ("ring", "bfloat16", 1 << 20, False, False),
    ("ring", "float32", (1 << 18) + 32, False, False),
    ("rhd", "bfloat16", 1 << 20, False, False),
    ("nvls", "bfloat16", 1 << 21, True, "ulp1"),
    ("nvls", "float32", 1 << 20, False, "ulp1"),
    ("nvls", "bfloat16", (1 << 20) + 64, False, "ulp1"),
    ("nvls", "float16", 1 << 20, False, "ulp1"),
    ("nvls_oneshot", "bfloat16", 1 << 14, False, False),
    ("ll", "bfloat16", 1000, False, True),
    ("ll", "float32", 1 << 16, False, True),
    ("ll", "bfloat16", 1 << 17, False, True),
    ("compressed", "bfloat16", (1 << 20) + 48, False, True),
    ("compressed_mc", "bfloat16", 1 << 21, False, True),
    ("compressed", "float32", 300_000, False, True),
    ("compressed_hybrid", "bfloat16", (1 << 20) + 48, False, True),
    ("compressed_hybrid_mc", "float16", 1 << 21, False, True),
    ("ce", "bfloat16", 1 << 20, False, True),
    ("ce_sym", "bfloat16", (1 << 22) + 64, True, True),
    ("ce_sym", "float32", 1 << 20, True, True),
]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_native_allreduce(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cases = [c for c in CASES if not (c[0] == "rhd" and world & (world - 1))]
    res = run_ranks(_worker, world, backend="nccl", args=(cases,), timeout=600,
                    env={"NCCL_DEBUG": "WARN"})
    bad = [r for rank_res in res for r in rank_res if r[-1] not in ("ok", "skipped-no-multicast")]
    assert not bad, bad
