"""GPU LZC1 codec kernels: bit-identical streams to the CPU oracle, lossless
round trips, slotted records, corruption reported through a status word."""
import pytest
import torch

from results_b200.ops import codec

pytestmark = pytest.mark.gpu


def _rand(n, dtype, std=0.02, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * std).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.uint8])
@pytest.mark.parametrize("n", [1, 15, 16, 1000, 32768, 32769, 300_007])
def test_gpu_stream_matches_cpu_oracle(dtype, n):
    if dtype == torch.uint8:
        x = torch.randint(0, 40, (n,), dtype=torch.uint8)
    else:
        x = _rand(n, dtype, seed=n)
    ref = codec.encode_cpu(x)
    got = codec.encode(x.cuda()).cpu()
    assert got.numel() == ref.numel()
    assert torch.equal(got, ref), "GPU stream differs from the CPU oracle"
    y = codec.decode(got.cuda(), n=n, dtype=dtype)
    assert torch.equal(y.cpu().view(torch.uint8), x.view(torch.uint8))


@pytest.mark.parametrize("kind", ["zeros", "uniform", "specials"])
def test_gpu_edge_distributions(kind):
    n = 100_000
    if kind == "zeros":
        x = torch.zeros(n, dtype=torch.bfloat16)
    elif kind == "uniform":
        x = torch.randint(-32768, 32767, (n,), dtype=torch.int16).view(torch.bfloat16)
    else:
        x = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0, -0.0, 1e-40, 3.0] * (n // 7),
                         dtype=torch.float32).to(torch.bfloat16)
    ref = codec.encode_cpu(x)
    got = codec.encode(x.cuda()).cpu()
    assert torch.equal(got, ref)
    y = codec.decode(got.cuda(), like=x.cuda())
    assert torch.equal(y.cpu().view(torch.int16), x.view(torch.int16))


def test_gpu_large_ratio():
    n = 64 << 20  # 128 MB bf16 (> L2)
    x = (torch.randn(n, device="cuda") * 0.02).to(torch.bfloat16)
    blob = codec.encode(x)
    y = codec.decode(blob, like=x)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    ratio = blob.numel() / (2 * n)
    assert 0.6 < ratio < 0.72, ratio


def test_slotted_roundtrip():
    x = (torch.randn(200_000, device="cuda") * 0.02).to(torch.bfloat16)
    slots, sizes = codec.encode_slotted(x)
    y = codec.decode_slotted(slots, x.numel(), x.dtype)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    assert int(sizes.max()) <= codec.tg_capacity(torch.bfloat16)


def test_gpu_corruption_reported_not_trapped():
    x = (torch.randn(100_000, device="cuda") * 0.02).to(torch.bfloat16)
    blob = codec.encode(x)
    bad = blob.clone()
    bad[64 + 8 * 4 + 3] ^= 0x11  # inside the TG offset table / first record header
    with pytest.raises(codec.CodecError):
        codec.decode(bad, like=x)
    bad2 = blob.clone()
    bad2[: 4] = 0  # stream magic
    with pytest.raises(codec.CodecError):
        codec.decode(bad2, like=x)
    # the context is still healthy afterwards
    y = codec.decode(blob, like=x)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
