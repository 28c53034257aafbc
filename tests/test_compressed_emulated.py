"""Fused compressed allreduce kernel on one GPU with R emulated ranks (one
cooperative launch): bit-identical to the fp32 rank-order reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def worlds():
    from results_b200.parallel.emulate import EmulatedWorld

    ws = {R: EmulatedWorld(R, heap_bytes=(160 << 20), stage_bytes=(96 << 20)) for R in (2, 4)}
    yield ws
    for w in ws.values():
        w.close()


def _inputs(R, n, dtype, seed, kind="grad"):
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = []
    for r in range(R):
        if kind == "grad":
            x = torch.randn(n, device="cuda", generator=g) * 1e-3
        else:  # activation-like with 1% outliers x50
            x = torch.randn(n, device="cuda", generator=g)
            m = torch.rand(n, device="cuda", generator=g) < 0.01
            x = torch.where(m, x * 50, x)
        xs.append(x.to(dtype))
    return xs


@pytest.mark.parametrize("level", ["ans", "pack"])
@pytest.mark.parametrize("hybrid", [False, True])
@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [16, 1000, 32768 * 3 + 48, 400_000, 400_001])
def test_compressed_allreduce_bitexact(worlds, R, dtype, n, hybrid, level):
    """hybrid=True: raw reduce-scatter, compressed all-gather; level: codec
    level of the records (rANS or PACK table codes)."""
    w = worlds[R]
    xs = _inputs(R, n, dtype, seed=n + R)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(2):
        w.compressed_allreduce(xs, outs, nblocks=8, hybrid=hybrid, level=level)
    torch.cuda.synchronize()
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()
    ref = acc.to(dtype)
    for r in range(R):
        assert w.status(r) == 0
        assert torch.equal(outs[r].view(torch.uint8), ref.view(torch.uint8)), f"rank {r}"


@pytest.mark.parametrize("level", ["ans", "pack"])
def test_compressed_inplace_activation_like(worlds, level):
    R = 4
    w = worlds[R]
    n = 300_000
    bufs = w.empty(n, torch.bfloat16)
    xs = _inputs(R, n, torch.bfloat16, seed=5, kind="act")
    for r in range(R):
        bufs[r].copy_(xs[r])
    w.compressed_allreduce(bufs, bufs, nblocks=16, level=level)
    torch.cuda.synchronize()
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()
    for r in range(R):
        assert torch.equal(bufs[r], acc.to(torch.bfloat16))


@pytest.mark.parametrize("level", ["ans", "pack"])
@pytest.mark.parametrize("hybrid", [False, True])
@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("chunk_tgs,nblocks", [(1, 1), (2, 2), (3, 2), (5, 3)])
def test_compressed_allreduce_chunked_ring(worlds, R, hybrid, level, chunk_tgs, nblocks):
    """In-launch chunks through a ring of two chunks' slots: slices of 13 table
    groups in chunks of 1-6 TGs (rounded up to the grid), 3 to 13 chunks, three
    calls in a row (progress flags are cleared per call), bit-exact."""
    w = worlds[R]
    n = 32768 * R * 12 + 48 * R + 16
    outs = None
    for it in range(3):
        xs = _inputs(R, n, torch.bfloat16, seed=1000 * it + 10 * R + chunk_tgs)
        outs = [torch.empty_like(x) for x in xs]
        w.compressed_allreduce(xs, outs, nblocks=nblocks, hybrid=hybrid, level=level,
                               chunk_elems=32768 * R * chunk_tgs)
        torch.cuda.synchronize()
        acc = xs[0].float().clone()
        for x in xs[1:]:
            acc += x.float()
        ref = acc.to(torch.bfloat16)
        for r in range(R):
            assert w.status(r) == 0
            assert torch.equal(outs[r].view(torch.uint8), ref.view(torch.uint8)), (it, r)


def test_chunked_stage_is_bounded():
    from results_b200.parallel import compressed as cz

    n = 256 << 20  # 512 MiB of bf16
    whole = cz.stage_bytes_needed(n, torch.bfloat16, 8, 444)
    chunked = cz.stage_bytes_needed(n, torch.bfloat16, 8, 444, chunk_elems=(64 << 20) // 2)
    assert chunked < whole / 3


@pytest.mark.parametrize("level", ["ans", "pack"])
@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("chunk", [0, 2])
def test_compressed_allreduce_stage_local(worlds, R, level, chunk):
    """Reduce-scatter records encoded locally and pushed as vectors, with and
    without chunks: same bit-exact result."""
    w = worlds[R]
    n = 32768 * R * 7 + 1000
    xs = _inputs(R, n, torch.float16, seed=77 + R)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(2):
        w.compressed_allreduce(xs, outs, nblocks=4, level=level, chunk_elems=32768 * R * chunk,
                               stage_local=True)
    torch.cuda.synchronize()
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()
    ref = acc.to(torch.float16)
    for r in range(R):
        assert w.status(r) == 0
        assert torch.equal(outs[r], ref), r


@pytest.mark.parametrize("R", [2, 4])
def test_compressed_allreduce_phase_tracer(worlds, R):
    """The per-CTA phase tracer: every table group of every slice is reduced by
    exactly one CTA, phase times are positive and their sum stays within the
    CTA's total."""
    from results_b200.parallel import compressed as cz

    w = worlds[R]
    G = 4
    n = 32768 * R * 5 + 100
    xs = _inputs(R, n, torch.bfloat16, seed=3)
    outs = [torch.empty_like(x) for x in xs]
    tr = torch.zeros((R, G, len(cz.TRACE_PHASES)), dtype=torch.int64, device="cuda")
    w.compressed_allreduce(xs, outs, nblocks=G, level="pack", trace=tr)
    torch.cuda.synchronize()
    slice_elems = ((n + R - 1) // R + 15) // 16 * 16
    tgs = [min(slice_elems, max(0, n - r * slice_elems)) for r in range(R)]
    tgs = sum((t + 32767) // 32768 for t in tgs)
    t = tr.cpu()
    assert int(t[:, :, cz.TRACE_PHASES.index("tgs_reduced")].sum()) == tgs
    total = t[:, :, 0]
    parts = t[:, :, 1:cz.TRACE_PHASES.index("tgs_reduced")].sum(dim=2)
    assert bool((total > 0).all()) and bool((parts <= total).all())
    assert int(t[:, :, cz.TRACE_PHASES.index("rs_encode_push")].sum()) > 0
    s = cz.summarize_trace(tr.view(R * G, -1))
    assert s["total"] > 0 and set(s) == set(cz.TRACE_PHASES)
