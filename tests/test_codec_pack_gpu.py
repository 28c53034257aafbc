"""PACK level of the GPU codec kernels: streams byte-identical to the CPU
oracle for every dtype and length class, lossless round trips, decoding of
records mixed with ANS streams, and corruption reported through the status
word."""
import pytest
import torch

from results_b200.ops import codec

pytestmark = pytest.mark.gpu


def _rand(n, dtype, std=0.02, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * std).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.uint8,
                                   torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("n", [1, 15, 16, 31, 33, 1000, 32768, 32769, 300_007])
def test_pack_gpu_matches_cpu_oracle(dtype, n):
    if dtype == torch.uint8:
        x = torch.randint(0, 40, (n,), dtype=torch.uint8)
    elif dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        x = _rand(n + (n & 1), torch.float32, std=0.5, seed=n).to(dtype)
    else:
        x = _rand(n, dtype, seed=n)
    ref = codec.encode_cpu(x, level="pack")
    got = codec.encode(x.cuda(), level="pack").cpu()
    assert got.numel() == ref.numel()
    assert torch.equal(got, ref), "GPU PACK stream differs from the CPU oracle"
    y = codec.decode(got.cuda(), n=x.numel(), dtype=dtype)
    assert torch.equal(y.cpu().view(torch.uint8), x.view(torch.uint8))


@pytest.mark.parametrize("kind", ["zeros", "uniform", "specials", "outliers", "two_symbols"])
def test_pack_gpu_edge_distributions(kind):
    n = 100_000
    g = torch.Generator().manual_seed(2)
    if kind == "zeros":
        x = torch.zeros(n, dtype=torch.bfloat16)
    elif kind == "uniform":
        x = torch.randint(-32768, 32767, (n,), generator=g, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    elif kind == "specials":
        x = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0, -0.0, 1e-40, 3.0] * (n // 7),
                         dtype=torch.float32).to(torch.bfloat16)
    elif kind == "outliers":
        v = torch.randn(n, generator=g)
        x = torch.where(torch.rand(n, generator=g) < 0.01, v * 50, v).to(torch.bfloat16)
    else:
        x = torch.where(torch.rand(n, generator=g) < 0.5, 1.0, 0.25).to(torch.bfloat16)
    ref = codec.encode_cpu(x, level="pack")
    got = codec.encode(x.cuda(), level="pack").cpu()
    assert torch.equal(got, ref)
    y = codec.decode(got.cuda(), like=x.cuda())
    assert torch.equal(y.cpu().view(torch.int16), x.view(torch.int16))


def test_pack_gpu_large_ratio_and_slotted():
    n = 64 << 20  # 128 MB bf16 (> L2)
    x = (torch.randn(n, device="cuda") * 0.02).to(torch.bfloat16)
    blob = codec.encode(x, level="pack")
    y = codec.decode(blob, like=x)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    assert 0.68 < blob.numel() / (2 * n) < 0.72
    slots, sizes = codec.encode_slotted(x[:300_000], level="pack")
    z = codec.decode_slotted(slots, 300_000, torch.bfloat16)
    assert torch.equal(z.view(torch.int16), x[:300_000].view(torch.int16))


def test_pack_gpu_corruption_reported():
    x = _rand(100_000, torch.bfloat16, seed=4)
    blob = codec.encode(x.cuda(), level="pack")
    rec0 = int(blob[64:72].cpu().view(torch.int64).item())
    for pos, val in ((rec0 + 22, 9), (rec0 + 28, 0)):  # code width, escape count
        bad = blob.clone()
        bad[pos] = val
        with pytest.raises(codec.CodecError):
            codec.decode(bad, like=x.cuda())
