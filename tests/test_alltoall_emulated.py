"""All-to-all kernel (raw zero-copy, raw via slots, split+rANS or split+PACK compressed)
with R ranks emulated on ONE GPU in one cooperative launch; every output
chunk must equal the matching input chunk of its source rank bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _expect(ins, R):
    chunks = [x.view(R, -1) for x in ins]
    return [torch.cat([chunks[src][r] for src in range(R)]) for r in range(R)]


@pytest.mark.parametrize("R", [2, 4, 8])
@pytest.mark.parametrize("mode", ["raw_slots", "raw_symmetric", "compressed", "compressed_pack"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_emulated_all_to_all(R, mode, dtype):
    from results_b200.parallel.emulate import EmulatedWorld

    w = EmulatedWorld(R, heap_bytes=(160 << 20), stage_bytes=(64 << 20))
    try:
        chunk = 40000 + 8 * R  # not a multiple of the 32768-element table group
        n = chunk * R
        for it in range(3):
            g = torch.Generator(device="cuda").manual_seed(17 * it + R)
            ins = [(torch.randn(n, device="cuda", generator=g) * 0.02).to(dtype) for _ in range(R)]
            if mode == "raw_symmetric":
                outs = w.empty(n, dtype)
            else:
                outs = [torch.full((n,), 7.0, device="cuda", dtype=dtype) for _ in range(R)]
            comp = {"compressed": True, "compressed_pack": "pack"}.get(mode, False)
            w.all_to_all(ins, outs, compress=comp, nblocks=4)
            torch.cuda.synchronize()
            for r, ref in enumerate(_expect(ins, R)):
                assert w.status(r) == 0
                assert torch.equal(outs[r].view(torch.uint8), ref.view(torch.uint8)), (it, r)
    finally:
        w.close()


def test_emulated_all_to_all_bytes():
    """uint8 payloads (raw only)."""
    from results_b200.parallel.emulate import EmulatedWorld

    R = 4
    w = EmulatedWorld(R, heap_bytes=(96 << 20), stage_bytes=(32 << 20))
    try:
        n = 4096 * R
        ins = [torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda") for _ in range(R)]
        outs = [torch.zeros(n, dtype=torch.uint8, device="cuda") for _ in range(R)]
        w.all_to_all(ins, outs)
        torch.cuda.synchronize()
        for r, ref in enumerate(_expect(ins, R)):
            assert torch.equal(outs[r], ref)
    finally:
        w.close()
