"""fp8 pair packers (CPU oracle): exhaustive round trip over all 65,536 byte
pairs, the reference's e4m3 container layout, the e5m2 bit-field encoder, and
fp8 codec round trips."""
import itertools

import pytest
import torch

from results_b200.ops import codec, fp8


def _all_pairs():
    a = torch.arange(256, dtype=torch.int32).repeat_interleave(256)
    b = torch.arange(256, dtype=torch.int32).repeat(256)
    return torch.stack([a, b], 1).reshape(-1).to(torch.uint8)


@pytest.mark.parametrize("kind", ["e4m3", "e5m2"])
def test_exhaustive_roundtrip(kind):
    x = _all_pairs()
    w = fp8.pack_fp8(x, kind)
    assert w.numel() == 65536
    assert len(set(w.view(torch.int16).tolist())) == 65536  # the container is a bijection
    y = fp8.unpack_fp8(w, kind)
    assert torch.equal(x, y)


def test_e4m3_reference_layout():
    # a = sign 1, exp 0b1010, mant 0b011 ; b = sign 0, exp 0b0101, mant 0b110
    a = (1 << 7) | (0b1010 << 3) | 0b011
    b = (0 << 7) | (0b0101 << 3) | 0b110
    w = int(fp8.pack_fp8(torch.tensor([a, b], dtype=torch.uint8), "e4m3").view(torch.int16)[0]) & 0xFFFF
    expect = (1 << 15) | (0b1010 << 11) | (0b0101 << 7) | (0b011 << 4) | (0 << 3) | 0b110
    assert w == expect
    # bits 14..7 (the bf16 exponent byte) hold both exponents
    assert (w >> 7) & 0xFF == (0b1010 << 4) | 0b0101


def test_e5m2_field_encoder_matches_torch_cast():
    vals = [0.0, -0.0, 1.0, -2.5, 3.14159, 1e-5, 6e-5, 57344.0, 1e6, -1e-8, 0.1, 448.0, float("inf"),
            float("-inf")]
    vals += [x / 7.0 for x in range(-300, 300)]
    t = torch.tensor(vals, dtype=torch.float32).to(torch.float8_e5m2).view(torch.uint8)
    for v, ref in zip(vals, t.tolist()):
        assert fp8.e5m2_byte(v) == ref, (v, fp8.e5m2_fields(v), ref)


@pytest.mark.parametrize("dt", [torch.float8_e4m3fn, torch.float8_e5m2])
def test_fp8_codec_roundtrip(dt):
    x = (torch.randn(100_002, generator=torch.Generator().manual_seed(2)) * 0.5).to(dt)
    blob = codec.encode_cpu(x)
    y = codec.decode_cpu(blob, x.numel(), dt)
    assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
    assert blob.numel() < 0.9 * x.numel()
    odd = x[:-1]  # odd length falls back to byte symbols
    y2 = codec.decode_cpu(codec.encode_cpu(odd), odd.numel(), dt)
    assert torch.equal(odd.view(torch.uint8), y2.view(torch.uint8))
