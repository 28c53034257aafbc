"""Weight-transfer kernel (K-slot credit pipeline, grouped work items,
split+rANS or raw) with sender and receivers emulated on ONE GPU in one
cooperative launch. Repeated transfers of changing data catch stale-slot
reads; receivers must end bit-identical to the sender."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def world3():
    from results_b200.parallel.emulate import EmulatedWorld

    w = EmulatedWorld(3, heap_bytes=(640 << 20), stage_bytes=(512 << 20))
    yield w
    w.close()


def _tensors(seed, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    shapes = [(1000, 512), (512,), (3, 32768), (77, 129), (70000,)]
    out = [(torch.randn(s, device=device, generator=g) * 0.02).to(torch.bfloat16) for s in shapes]
    out.append((torch.randn(50000, device=device, generator=g)).to(torch.float32))
    out.append((torch.randn(40000, device=device, generator=g) * 0.5).to(torch.float8_e4m3fn))
    return out


@pytest.mark.parametrize("encode", [1, 0, 2])  # split + rANS, raw, split + PACK codes
@pytest.mark.parametrize("bcast", [False, True])
def test_emulated_transfer_repeated(world3, encode, bcast):
    R = 3
    for it in range(4):
        src_t = _tensors(100 * it + int(encode) + 3 * int(bcast))
        recv = {r: [torch.full_like(t, 0) for t in src_t] for r in (1, 2)}
        tensors = [src_t, recv[1], recv[2]]
        if bcast:
            world3.weight_transfer(0, [1, 2], tensors, encode=encode, broadcast_all=True)
        else:
            for d in (1, 2):
                world3.weight_transfer(0, [d], tensors, encode=encode)
        torch.cuda.synchronize()
        for r in (1, 2):
            assert world3.status(r) == 0
            for a, b in zip(recv[r], src_t):
                assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), (it, r, a.shape)


@pytest.mark.parametrize("src", [0, 2])
def test_emulated_relay_broadcast(src):
    """Relay broadcast: chunks dealt to owner ranks that forward them; every
    rank's symmetric tensors must end bit-identical to the sender's source,
    over repeated calls with changing data and a sender whose source is not
    its own destination."""
    from results_b200.parallel.emulate import EmulatedWorld

    R = 4
    w = EmulatedWorld(R, heap_bytes=(256 << 20))
    try:
        shapes = [(1000, 512), (7,), (3, 32768), (77, 129), (700001,), (1 << 20,)]
        dst = [w.empty(s, torch.bfloat16) for s in shapes]  # dst[i][r]
        per_rank = [[dst[i][r] for i in range(len(shapes))] for r in range(R)]
        for it in range(3):
            g = torch.Generator(device="cuda").manual_seed(1000 * it + src)
            srcs = [(torch.randn(s, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for s in shapes]
            for r in range(R):
                for t in per_rank[r]:
                    t.fill_(float(r + 1))
            w.broadcast_relay(src, per_rank, srcs, nblocks=6)
            torch.cuda.synchronize()
            for r in range(R):
                assert w.status(r) == 0
                for a, b in zip(per_rank[r], srcs):
                    assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), (it, r, a.shape)
    finally:
        w.close()
