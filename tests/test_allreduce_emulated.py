"""Multi-rank allreduce kernels on ONE GPU: R emulated ranks in one cooperative
launch (the same kernel bodies as the NVLink path). Compared element-wise with
a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def _inputs(R, n, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [(torch.randn(n, device="cuda", generator=g) * 1e-2 * (r + 1)).to(dtype) for r in range(R)]


def _ref(xs):
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()  # rank order, fp32
    return acc.to(xs[0].dtype)


@pytest.fixture(scope="module")
def emu_worlds():
    from results_b200.parallel.emulate import EmulatedWorld

    ws = {R: EmulatedWorld(R, heap_bytes=192 << 20, stage_bytes=64 << 20) for R in (2, 4, 8)}
    yield ws
    for w in ws.values():
        w.close()


@pytest.mark.parametrize("R", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [8, 1000, 4096, 1 << 18])
def test_oneshot_bitexact(emu_worlds, R, dtype, n):
    w = emu_worlds[R]
    xs = _inputs(R, n, dtype, seed=n + R)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(3):  # repeated calls exercise the double-buffered stage
        w.allreduce(xs, outs, "oneshot", nblocks=8, nthreads=256)
    torch.cuda.synchronize()
    ref = _ref(xs)
    for r in range(R):
        assert w.status(r) == 0
        assert torch.equal(outs[r], ref), f"rank {r} differs"


@pytest.mark.parametrize("R", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [8, 1000, 4096, 1 << 16])
def test_ll_bitexact(emu_worlds, R, dtype, n):
    """Low-latency one-shot: flag-in-data words, parity areas reused across
    calls (interleaved with one-shot so the call parity moves on)."""
    w = emu_worlds[R]
    es = torch.empty((), dtype=dtype).element_size()
    if (n * es) % 16:
        pytest.skip("ll needs a multiple of 16 bytes")
    ref = None
    for it in range(5):
        xs = _inputs(R, n, dtype, seed=n + R + it)
        outs = [torch.empty_like(x) for x in xs]
        w.allreduce(xs, outs, "ll" if it != 2 else "oneshot", nblocks=8, nthreads=256)
        torch.cuda.synchronize()
        ref = _ref(xs)
        for r in range(R):
            assert w.status(r) == 0
            assert torch.equal(outs[r], ref), f"call {it} rank {r} differs"


@pytest.mark.parametrize("R", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1024, 1 << 16, (1 << 20) + 64])
def test_twoshot_bitexact(emu_worlds, R, dtype, n):
    w = emu_worlds[R]
    xs = _inputs(R, n, dtype, seed=7 * n + R)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(2):
        w.allreduce(xs, outs, "twoshot", nblocks=16, nthreads=256)
    torch.cuda.synchronize()
    ref = _ref(xs)
    for r in range(R):
        assert w.status(r) == 0
        assert torch.equal(outs[r], ref), f"rank {r} differs"


@pytest.mark.parametrize("R", [2, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_twoshot_symmetric_inplace(emu_worlds, R, dtype):
    w = emu_worlds[R]
    n = (1 << 18) + 8 * 3
    bufs = w.empty(n, dtype)
    xs = _inputs(R, n, dtype, seed=3)
    for r in range(R):
        bufs[r].copy_(xs[r])
    w.allreduce(bufs, bufs, "twoshot", nblocks=16, nthreads=256)
    torch.cuda.synchronize()
    ref = _ref(xs)
    for r in range(R):
        assert torch.equal(bufs[r], ref)


@pytest.mark.parametrize("R", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [4096, (1 << 19) + 8 * 5])
def test_ring(emu_worlds, R, dtype, n):
    w = emu_worlds[R]
    xs = _inputs(R, n, dtype, seed=11 * n + R)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(2):
        w.allreduce(xs, outs, "ring", nblocks=4, nthreads=128)
    torch.cuda.synchronize()
    ref = torch.stack([x.float() for x in xs]).sum(0)
    tol = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-2}[dtype]
    for r in range(R):
        assert w.status(r) == 0
        torch.testing.assert_close(outs[r].float(), ref, atol=tol * ref.abs().max().item(), rtol=tol)
    # every rank holds the same values
    for r in range(1, R):
        assert torch.equal(outs[r], outs[0])


@pytest.mark.parametrize("R", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [4096, (1 << 19) + 8 * 5])
def test_rhd(emu_worlds, R, dtype, n):
    w = emu_worlds[R]
    xs = _inputs(R, n, dtype, seed=13 * n + R)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(2):
        w.allreduce(xs, outs, "rhd", nblocks=8, nthreads=256)
    torch.cuda.synchronize()
    ref = torch.stack([x.float() for x in xs]).sum(0)
    tol = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-2}[dtype]
    for r in range(R):
        assert w.status(r) == 0
        torch.testing.assert_close(outs[r].float(), ref, atol=tol * ref.abs().max().item(), rtol=tol)
    for r in range(1, R):
        assert torch.equal(outs[r], outs[0])


def test_mixed_algorithms_sequence(emu_worlds):
    """Different algorithms and grid sizes back to back on one communicator."""
    R = 4
    w = emu_worlds[R]
    for i, (algo, nb, n) in enumerate([("oneshot", 4, 5000), ("twoshot", 16, 1 << 16),
                                       ("ring", 2, 1 << 15), ("oneshot", 12, 64),
                                       ("rhd", 6, 1 << 14), ("twoshot", 3, 1 << 12)]):
        xs = _inputs(R, n, torch.float32, seed=i)
        outs = [torch.empty_like(x) for x in xs]
        w.allreduce(xs, outs, algo, nblocks=nb, nthreads=256)
        ref = torch.stack(xs).sum(0)
        for r in range(R):
            torch.testing.assert_close(outs[r], ref, atol=1e-5, rtol=1e-5)
