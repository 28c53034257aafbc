"""PACK level of the LZC1 codec on the CPU oracle: lossless round trips, the
record layout checked byte for byte against an independent Python statement
of the format, validation of corrupt records, and the measured ratio."""
import struct

import numpy as np
import pytest
import torch

from results_b200.ops import codec


def _rand(n, dtype, std=0.02, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * std).to(dtype)


def _header(rec):
    f = struct.unpack("<IHBBIIIHHII", bytes(rec[:32].tolist()))
    keys = ("magic", "version", "mode", "dtype", "n", "sym_bytes", "raw_bytes", "nnz", "nsub", "total", "reserved")
    return dict(zip(keys, f))


def _pad16(x):
    return (x + 15) // 16 * 16


def _py_pack_section(syms: np.ndarray):
    """Symbol section of a PACK record from the format description alone
    (csrc/lz_codec_format.h), or None when RAW is smaller."""
    n = len(syms)
    counts = np.bincount(syms, minlength=256)
    order = sorted(range(256), key=lambda s: (-counts[s], s))
    top = [s for s in order[:15] if counts[s]]
    best = (None, _pad16(n))
    if len(top) == 1 and counts[top[0]] == n and 16 < best[1]:
        best = (0, 16)
    groups = (n + 31) // 32
    for b in range(1, 5):
        k = min((1 << b) - 1, len(top))
        nesc = n - int(sum(counts[s] for s in top[:k]))
        if nesc * 16 > n:  # at most one escaped symbol in 16
            continue
        size = 16 + _pad16(groups * 4 * b) + _pad16(nesc)
        if size < best[1]:
            best = (b, size)
    b, size = best
    if b is None:
        return None
    nnz = 1 if b == 0 else min((1 << b) - 1, len(top))
    table = bytes(top[:nnz]) + bytes(16 - nnz)
    if b == 0:
        return b, nnz, 0, table
    esc = (1 << b) - 1
    code_of = {s: c for c, s in enumerate(top[:nnz])}
    codes = bytearray(_pad16(groups * 4 * b))
    escs = bytearray()
    for i, s in enumerate(syms.tolist()):
        c = code_of.get(s, esc)
        if c == esc:
            escs.append(s)
        bit = (i // 32) * 32 * b + (i % 32) * b
        for q in range(b):
            if (c >> q) & 1:
                codes[(bit + q) >> 3] |= 1 << ((bit + q) & 7)
    nesc = len(escs)
    escs += bytes(_pad16(nesc) - nesc)
    return b, nnz, nesc, table + bytes(codes) + bytes(escs)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [0, 1, 7, 16, 31, 33, 1000, 32768, 32769, 100_003])
def test_pack_roundtrip_bitexact(dtype, n):
    x = _rand(n, dtype, seed=n + 11)
    blob = codec.encode_cpu(x, level="pack")
    y = codec.decode_cpu(blob, n, dtype)
    assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))


@pytest.mark.parametrize("kind", ["zeros", "const", "uniform_bytes", "specials", "outliers", "few_symbols"])
def test_pack_edge_distributions(kind):
    n = 70_000
    g = torch.Generator().manual_seed(3)
    if kind == "zeros":
        x = torch.zeros(n, dtype=torch.bfloat16)
    elif kind == "const":
        x = torch.full((n,), 3.25, dtype=torch.bfloat16)
    elif kind == "uniform_bytes":
        x = torch.randint(0, 65536, (n,), generator=g, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    elif kind == "specials":
        x = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0, -0.0, 1e-40] * (n // 6),
                         dtype=torch.float32).to(torch.bfloat16)
    elif kind == "outliers":  # activation-like: N(0, 1) with 1 % outliers x 50
        v = torch.randn(n, generator=g)
        m = torch.rand(n, generator=g) < 0.01
        x = torch.where(m, v * 50, v).to(torch.bfloat16)
    else:  # two distinct symbols: a partial table (codes 2..esc-1 unused)
        x = torch.where(torch.rand(n, generator=g) < 0.5, 1.0, 0.25).to(torch.bfloat16)
    blob = codec.encode_cpu(x, level="pack")
    y = codec.decode_cpu(blob, x.numel(), x.dtype)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))


def test_pack_record_matches_format_statement():
    for seed, (n, std) in enumerate([(32768, 0.02), (5000, 1.0), (32768, 1e-3), (100, 0.5)]):
        x = _rand(n, torch.bfloat16, std=std, seed=seed)
        rec = codec.tg_encode_cpu(x, level="pack")
        h = _header(rec)
        u = x.view(torch.int16).numpy().astype(np.uint16)
        syms = ((u >> 7) & 0xFF).astype(np.uint8)
        exp = _py_pack_section(syms)
        assert exp is not None and h["mode"] == 2, (seed, h)
        b, nnz, nesc, section = exp
        assert (h["nsub"], h["nnz"], h["reserved"], h["sym_bytes"]) == (b, nnz, nesc, len(section))
        off = 32 + h["raw_bytes"]
        assert bytes(rec[off:off + len(section)].tolist()) == section, seed
        assert h["total"] == rec.numel() == off + len(section)


def test_pack_constant_uses_zero_bit_codes():
    x = torch.full((32768,), -2.0, dtype=torch.bfloat16)
    h = _header(codec.tg_encode_cpu(x, level="pack"))
    assert (h["mode"], h["nsub"], h["nnz"], h["sym_bytes"]) == (2, 0, 1, 16)


def test_pack_incompressible_falls_back_to_raw():
    g = torch.Generator().manual_seed(4)
    x = torch.randint(0, 65536, (32768,), generator=g, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    assert _header(codec.tg_encode_cpu(x, level="pack"))["mode"] == 0


def test_pack_ratio_bf16_16M_normal():
    """16M-element N(0, 0.02) bf16: 3-bit codes, ~4 % escapes."""
    n = 16 * 1024 * 1024
    x = _rand(n, torch.bfloat16, std=0.02, seed=0)
    blob = codec.encode_cpu(x, level="pack")
    y = codec.decode_cpu(blob, n, torch.bfloat16)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    ratio = blob.numel() / (2 * n)
    ans = codec.encode_cpu(x).numel() / (2 * n)
    assert 0.68 < ratio < 0.74, ratio
    assert ans < ratio


def test_pack_corrupt_records_rejected():
    x = _rand(32768, torch.bfloat16, seed=21)
    rec = codec.tg_encode_cpu(x, level="pack")
    h = _header(rec)
    assert h["mode"] == 2 and h["reserved"] > 0

    def patched(field_off, fmt, value):
        bad = rec.clone()
        bad[field_off:field_off + struct.calcsize(fmt)] = torch.tensor(list(struct.pack(fmt, value)), dtype=torch.uint8)
        return bad

    for bad in (patched(28, "<I", h["reserved"] + 1),   # escape count
                patched(22, "<H", 7),                     # code width
                patched(20, "<H", 0)):                    # table size
        with pytest.raises(codec.CodecError):
            codec.tg_decode_cpu(bad, x.numel(), x.dtype)
    # an escape code where the stream holds none: zero the escape count and the
    # escape section size follows, so the record size no longer matches
    with pytest.raises(codec.CodecError):
        codec.tg_decode_cpu(patched(28, "<I", 0), x.numel(), x.dtype)


def test_pack_invalid_code_in_partial_table_rejected():
    g = torch.Generator().manual_seed(8)
    x = torch.where(torch.rand(32768, generator=g) < 0.5, 1.0, 0.25).to(torch.bfloat16)
    rec = codec.tg_encode_cpu(x, level="pack")
    h = _header(rec)
    assert h["mode"] == 2 and h["nsub"] == 2 and h["nnz"] == 2  # codes 0, 1 used; 2 invalid; 3 escape
    codes = 32 + h["raw_bytes"] + 16
    bad = rec.clone()
    bad[codes] = (int(bad[codes]) & ~0x3) | 0x2  # element 0 gets code 2
    with pytest.raises(codec.CodecError):
        codec.tg_decode_cpu(bad, x.numel(), x.dtype)


def test_unknown_level_rejected():
    with pytest.raises(ValueError):
        codec.encode_cpu(_rand(10, torch.bfloat16), level="zstd")


def test_level_argument_encoding():
    """Host entry points take the encoder level in bits 8..11 of the dtype argument."""
    assert codec.level_code("ans") == 0 and codec.level_code("pack") == 1 and codec.level_code(1) == 1
    assert codec.with_level(2, "pack") == 2 | (1 << 8) and codec.with_level(0, "ans") == 0
    with pytest.raises(ValueError):
        codec.level_code(7)


def test_alltoall_compress_argument():
    from results_b200.parallel.alltoall import enc_code

    assert [enc_code(x) for x in (False, None, True, "ans", "pack")] == [0, 0, 1, 1, 2]
    with pytest.raises(ValueError):
        enc_code("zstd")


def test_trace_summary_means_per_cta_and_call():
    from results_b200.parallel import compressed as cz

    buf = torch.zeros((4, len(cz.TRACE_PHASES)), dtype=torch.int64)
    buf[:, 0] = 6000  # 6 us total per CTA over two calls
    buf[:, cz.TRACE_PHASES.index("reduce")] = torch.tensor([1000, 2000, 3000, 4000])
    buf[:, cz.TRACE_PHASES.index("tgs_reduced")] = 10
    s = cz.summarize_trace(buf, calls=2)
    assert s["total"] == 3.0 and s["reduce"] == 1.25 and s["tgs_reduced"] == 5.0


def test_pack_level_codes_raw_when_the_table_fits_badly():
    """fp16 N(0, 0.5): the high byte carries the sign, the top-15 table covers
    about 60 % of the symbols, so every width escapes more than one symbol in
    16 and the groups are coded RAW (still lossless)."""
    x = _rand(32768, torch.float16, std=0.5, seed=12)
    rec = codec.tg_encode_cpu(x, level="pack")
    assert _header(rec)["mode"] == 0
    y = codec.tg_decode_cpu(rec, x.numel(), x.dtype)
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))
