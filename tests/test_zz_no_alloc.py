"""Allocation-free codec entry point (lz_codec_encode_noalloc).

Callers that cannot allocate device memory when they compress -- e.g. a
serving process whose HBM budget is fixed at start-up, or a latency-critical
path that must avoid cudaMalloc's implicit synchronisation -- use this entry
point, which keeps its scratch in a fixed 32 MiB array inside the library.
The test calls it through its exported C symbol, twice in a row, and checks
that each stream is byte-identical to the one produced by the allocating
entry point (lz_codec_encode with caller scratch) and decodes losslessly.
The file name sorts last so a stop-at-first-failure run reaches it last.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_symbol():
    from results_b200 import _native

    lib = _native.cuda()  # the in-tree liblz_cuda.so
    f = lib.lz_codec_encode_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
    m = lib.lz_codec_noalloc_max_elems
    m.restype = C.c_size_t
    m.argtypes = [C.c_int]
    return lib, f, m


def _call(f, lib, x, dt):
    n = x.numel()
    cap = lib.lz_codec_max_bytes(n, dt)
    out = torch.empty(cap, dtype=torch.uint8, device="cuda")
    total = torch.zeros(1, dtype=torch.int64, device="cuda")
    rc = f(x.data_ptr(), n, dt, out.data_ptr(), cap, total.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.lz_last_error().decode()
    torch.cuda.synchronize()
    return out[: int(total.item())]


def test_noalloc_matches_allocating_encoder_two_calls():
    from results_b200.ops import codec

    lib, f, _ = _noalloc_symbol()
    cases = [(torch.bfloat16, 3_000_017, 11), (torch.float32, 1_234_567, 12)]
    for dtype, n, seed in cases:  # two calls in a row share the static scratch
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = (torch.randn(n, device="cuda", generator=g) * 0.02).to(dtype)
        got = _call(f, lib, x, codec.codec_dtype(dtype))
        ref = codec.encode(x)  # existing entry point, torch-allocated scratch
        assert got.numel() == ref.numel()
        assert torch.equal(got, ref), "noalloc stream differs from lz_codec_encode"
        y = codec.decode(got, like=x)
        assert torch.equal(y.view(torch.uint8), x.view(torch.uint8))


def test_noalloc_fp8_pair_dtypes_match_allocating_encoder():
    from results_b200.ops import codec

    lib, f, maxel = _noalloc_symbol()
    for name, seed in (("float8_e4m3fn", 21), ("float8_e5m2", 22)):
        fp8 = getattr(torch, name, None)
        if fp8 is None:
            continue
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = (torch.randn(2 * 700_001, device="cuda", generator=g) * 0.05).to(fp8)
        dt, n = codec.plan(x.dtype, x.numel())
        assert dt in (codec.DT_E4M3P, codec.DT_E5M2P) and maxel(dt) > n
        for _ in range(2):
            out = torch.empty(lib.lz_codec_max_bytes(n, dt), dtype=torch.uint8, device="cuda")
            total = torch.zeros(1, dtype=torch.int64, device="cuda")
            rc = f(x.view(torch.uint8).data_ptr(), n, dt, out.data_ptr(), out.numel(), total.data_ptr(),
                   torch.cuda.current_stream().cuda_stream)
            assert rc == 0, lib.lz_last_error().decode()
            torch.cuda.synchronize()
            got = out[: int(total.item())]
            ref = codec.encode(x)
            assert torch.equal(got, ref), f"noalloc {name} stream differs from lz_codec_encode"


def test_noalloc_rejects_inputs_beyond_the_fixed_scratch():
    from results_b200.ops import codec

    lib, f, maxel = _noalloc_symbol()
    dt = codec.codec_dtype(torch.bfloat16)
    limit = maxel(dt)
    assert limit > 16_000_000
    x = torch.empty(limit + 1, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(16, dtype=torch.uint8, device="cuda")
    total = torch.zeros(1, dtype=torch.int64, device="cuda")
    rc = f(x.data_ptr(), limit + 1, dt, out.data_ptr(), 16, total.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert "scratch" in lib.lz_last_error().decode()
