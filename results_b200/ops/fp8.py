"""fp8 e4m3 / e5m2 pair packing.

``pack_fp8(x)`` turns an fp8 tensor (or raw bytes) of even length into a
uint16 tensor of containers whose bits 14..7 -- the bf16 exponent byte --
hold exponent bits of both values of the pair, so the bf16 split codec codes
one symbol per two values. e4m3 uses the reference layout
(back_up/fp8_e4m3fn_pack_benchmark.cu:21-31); e5m2 (5+5 exponent bits do not fit
a byte) keeps the high four exponent bits of each value in the symbol byte.
The packers are also fused into the codec (``DT_E4M3P`` / ``DT_E5M2P``) so
weight transfers of fp8 tensors pack on the fly inside the sending kernel.

``e5m2_fields(x)`` is the pure-Python float -> e5m2 bit-field encoder of the
reference's demo (back_up/test.py:3-141), kept as a readable oracle.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from .. import _native, _native_sigs
from ..utils.trace import traced

_native_sigs.add_cuda({
    "lz_fp8_pack": (C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p),
    "lz_fp8_unpack": (C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p),
})

KINDS = {"e4m3": 0, "e5m2": 1}


def _kind(x_or_kind) -> int:
    if isinstance(x_or_kind, str):
        return KINDS[x_or_kind]
    if x_or_kind == getattr(torch, "float8_e5m2", None):
        return 1
    return 0


@traced("pack_fp8")
def pack_fp8(x: torch.Tensor, kind: str | None = None) -> torch.Tensor:
    """fp8 (or uint8) tensor of even length -> uint16 containers (one per pair)."""
    k = KINDS[kind] if kind else _kind(x.dtype)
    b = x.contiguous().view(torch.uint8).view(-1)
    if b.numel() % 2:
        raise ValueError("pack_fp8 needs an even number of values")
    npairs = b.numel() // 2
    out = torch.empty(npairs, dtype=torch.uint16 if hasattr(torch, "uint16") else torch.int16, device=b.device)
    if b.is_cuda:
        s = torch.cuda.current_stream(b.device).cuda_stream
        _native.check(_native.cuda().lz_fp8_pack(b.data_ptr(), out.data_ptr(), npairs, k, s), "fp8 pack")
    else:
        fn = _native.cpu().lz_cpu_pack_e4m3 if k == 0 else _native.cpu().lz_cpu_pack_e5m2
        fn(b.data_ptr(), out.data_ptr(), npairs)
    return out


@traced("unpack_fp8")
def unpack_fp8(w: torch.Tensor, kind: str = "e4m3", dtype: torch.dtype | None = None) -> torch.Tensor:
    """uint16 containers -> fp8 bytes (viewed as `dtype` when given)."""
    k = KINDS[kind]
    w = w.contiguous().view(-1)
    npairs = w.numel()
    out = torch.empty(2 * npairs, dtype=torch.uint8, device=w.device)
    if w.is_cuda:
        s = torch.cuda.current_stream(w.device).cuda_stream
        _native.check(_native.cuda().lz_fp8_unpack(w.data_ptr(), out.data_ptr(), npairs, k, s), "fp8 unpack")
    else:
        fn = _native.cpu().lz_cpu_unpack_e4m3 if k == 0 else _native.cpu().lz_cpu_unpack_e5m2
        fn(w.data_ptr(), out.data_ptr(), npairs)
    if dtype is not None:
        return out.view(dtype)
    return out


def e5m2_fields(x: float) -> tuple[int, int, int]:
    """(sign, biased exponent, mantissa) of the e5m2 encoding of x (bias 15),
    round-to-nearest-even, with subnormals, inf and nan."""
    sign = 1 if (x < 0 or (x == 0 and math.copysign(1.0, x) < 0)) else 0
    a = abs(x)
    if math.isnan(a):
        return sign, 31, 2
    if math.isinf(a):
        return sign, 31, 0
    if a == 0:
        return sign, 0, 0
    e = math.floor(math.log2(a))
    if e < -14:  # subnormal: value = m / 4 * 2^-14
        m = round(a / 2.0 ** -14 * 4)
        if m >= 4:
            return sign, 1, 0
        return sign, 0, m
    frac = a / 2.0 ** e - 1.0
    m = frac * 4
    mi = math.floor(m)
    rem = m - mi
    if rem > 0.5 or (rem == 0.5 and mi % 2 == 1):
        mi += 1
    if mi == 4:
        mi = 0
        e += 1
    if e + 15 >= 31:
        return sign, 31, 0  # overflow to inf
    return sign, e + 15, mi


def e5m2_byte(x: float) -> int:
    s, e, m = e5m2_fields(x)
    return (s << 7) | (e << 2) | m
