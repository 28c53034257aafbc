"""fp8 packing kernels and fp8 codec on the GPU, bit-identical to the CPU oracle."""
import pytest
import torch

from results_b200.ops import codec, fp8

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["e4m3", "e5m2"])
@pytest.mark.parametrize("n", [2, 30, 4096, 1_000_002])
def test_pack_unpack_matches_cpu(kind, n):
    g = torch.Generator().manual_seed(12345)
    x = torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g)
    w_cpu = fp8.pack_fp8(x, kind)
    w_gpu = fp8.pack_fp8(x.cuda(), kind)
    assert torch.equal(w_gpu.cpu().view(torch.int16), w_cpu.view(torch.int16))
    y = fp8.unpack_fp8(w_gpu, kind)
    assert torch.equal(y.cpu(), x)


@pytest.mark.parametrize("dt", [torch.float8_e4m3fn, torch.float8_e5m2])
def test_fp8_codec_gpu_matches_cpu(dt):
    x = (torch.randn(300_000, generator=torch.Generator().manual_seed(4)) * 0.5).to(dt)
    ref = codec.encode_cpu(x)
    got = codec.encode(x.cuda()).cpu()
    assert torch.equal(got, ref)
    y = codec.decode(got.cuda(), like=x.cuda())
    assert torch.equal(y.cpu().view(torch.uint8), x.view(torch.uint8))
