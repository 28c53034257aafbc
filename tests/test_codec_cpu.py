"""CPU oracle of the LZC1 codec: lossless round trips, format validation and
measured compression ratios (the CPU configuration: bf16 split round trip with a
reference CPU rANS of the exponent stream on 16M N(0, 0.02) elements)."""
import pytest
import torch

from results_b200.ops import codec


def _rand(n, dtype, std=0.02, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * std).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [0, 1, 7, 16, 1000, 32768, 32769, 100_003])
def test_roundtrip_bitexact(dtype, n):
    x = _rand(n, dtype, seed=n)
    blob = codec.encode_cpu(x)
    y = codec.decode_cpu(blob, n, dtype)
    assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))


@pytest.mark.parametrize("kind", ["zeros", "const", "uniform_bytes", "specials"])
def test_roundtrip_edge_distributions(kind):
    n = 70_000
    if kind == "zeros":
        x = torch.zeros(n, dtype=torch.bfloat16)
    elif kind == "const":
        x = torch.full((n,), 3.25, dtype=torch.bfloat16)
    elif kind == "uniform_bytes":  # incompressible symbol plane -> RAW table groups
        x = torch.randint(0, 65536, (n,), dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    else:
        x = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0, -0.0, 1e-40] * (n // 6),
                         dtype=torch.float32).to(torch.bfloat16)
    blob = codec.encode_cpu(x)
    y = codec.decode_cpu(blob, x.numel(), x.dtype)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    if kind == "uniform_bytes":
        assert blob.numel() <= x.numel() * 2 + 64 + 8 * 3 + 3 * 64  # never expands beyond headers


def test_uint8_and_fp8_roundtrip():
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(50_000, generator=g) * 0.5).to(torch.float8_e5m2)
    blob = codec.encode_cpu(x)
    y = codec.decode_cpu(blob, x.numel(), x.dtype)
    assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
    assert blob.numel() < x.numel()  # e5m2 bytes are compressible


def test_ratio_bf16_16M_normal():
    """16M-element N(0, 0.02) bf16 tensor, reference CPU rANS of the exponent stream."""
    n = 16 * 1024 * 1024
    x = _rand(n, torch.bfloat16, std=0.02, seed=0)
    blob = codec.encode_cpu(x)
    y = codec.decode_cpu(blob, n, torch.bfloat16)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    ratio = blob.numel() / (2 * n)
    # exponent entropy ~2.7 bits -> (8 + 2.7 + overheads) / 16 ~ 0.67-0.69
    assert 0.60 < ratio < 0.72, ratio
    h = codec.symbol_entropy_bits(x)
    assert ratio < (8 + h) / 16 + 0.03  # within 3 points of the order-0 entropy bound


def test_ratio_by_dtype_ordering():
    """bf16 compresses best, fp16/fp32 less (reference csv/compress_ratio.csv:7 ordering)."""
    n = 1 << 20
    r = {}
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        x = _rand(n, dt, seed=3)
        r[dt] = codec.encode_cpu(x).numel() / (n * x.element_size())
    assert r[torch.bfloat16] < r[torch.float16] and r[torch.bfloat16] < r[torch.float32]
    assert r[torch.float32] < 0.9 and r[torch.float16] < 0.95


def test_corrupt_stream_detected():
    x = _rand(40_000, torch.bfloat16, seed=5)
    blob = codec.encode_cpu(x)
    rec0 = int(blob[64:72].view(torch.int64).item())  # offset of the first table group
    raw_bytes = int(blob[rec0 + 16:rec0 + 20].view(torch.int32).item())
    ans = rec0 + 32 + raw_bytes
    # stream magic, TG offset, TG magic, TG size field, frequency table, lane states, words
    for pos in (0, 64, rec0, rec0 + 12, ans + 1, ans + 48 + 5, ans + 48 + 200):
        bad = blob.clone()
        bad[pos] ^= 0x5A
        try:
            y = codec.decode_cpu(bad, x.numel(), x.dtype)
        except codec.CodecError:
            continue
        assert not torch.equal(y.view(torch.int16), x.view(torch.int16)), pos
    with pytest.raises(codec.CodecError):
        codec.decode_cpu(blob[:100], x.numel(), x.dtype)


def test_tg_record_api():
    x = _rand(32768, torch.bfloat16, seed=9)
    rec = codec.tg_encode_cpu(x)
    assert rec.numel() % 16 == 0
    y = codec.tg_decode_cpu(rec, x.numel(), x.dtype)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))


def test_decode_from_fixed_size_padded_buffer():
    """A stream copied into a fixed-size message (the fixed-budget transfers
    of the compressed ring) decodes from its prefix; trailing bytes of the
    budget are ignored whatever they hold."""
    from results_b200.ops import codec

    torch.manual_seed(5)
    x = (torch.randn(300_000) * 0.02).to(torch.bfloat16)
    blob = codec.encode_cpu(x)
    budget = blob.numel() + 4096
    msg = torch.randint(0, 256, (budget,), dtype=torch.uint8)
    msg[: blob.numel()] = blob
    y = codec.decode_cpu(msg, x.numel(), x.dtype)
    assert torch.equal(y.view(torch.int16), x.view(torch.int16))


def test_cpu_stream_identical_for_any_thread_count():
    """The CPU oracle encodes table groups on several threads and packs them in
    order: the stream bytes do not depend on LZ_CPU_THREADS (a subprocess per
    setting, since the variable is read by the native library)."""
    import os
    import subprocess
    import sys

    code = ("import torch,hashlib\nfrom results_b200.ops import codec\n"
            "g=torch.Generator().manual_seed(3)\nx=(torch.randn(1_000_003,generator=g)*0.02).to(torch.bfloat16)\n"
            "b=codec.encode_cpu(x)\ny=codec.decode_cpu(b,x.numel(),x.dtype)\n"
            "assert torch.equal(x.view(torch.int16),y.view(torch.int16))\n"
            "print(hashlib.sha256(b.numpy().tobytes()).hexdigest())\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = set()
    for n in ("1", "3", "16"):
        env = dict(os.environ, LZ_CPU_THREADS=n, PYTHONPATH=root)
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, cwd=root)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.add(r.stdout.strip())
    assert len(outs) == 1


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 32767, 32768, 32769])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.uint8])
def test_roundtrip_edge_lengths(n, dtype):
    """Empty tensors, tails shorter than a 16-element unit and table-group
    boundaries round-trip bit-exactly."""
    x = _rand(n, dtype) if dtype != torch.uint8 else torch.randint(0, 256, (n,), dtype=torch.uint8)
    y = codec.decode_cpu(codec.encode_cpu(x), n, dtype)
    assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))


@pytest.mark.parametrize("n", [0, 1, 2, 3, 1001])
@pytest.mark.parametrize("dtype", [torch.float8_e4m3fn, torch.float8_e5m2])
def test_fp8_odd_lengths(n, dtype):
    """fp8 tensors with an odd element count (a half-filled last pair container)."""
    x = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 0.5).to(dtype)
    y = codec.decode_cpu(codec.encode_cpu(x), n, dtype)
    assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
