"""LZC1 lossless float codec: exponent-byte rANS + raw sign/mantissa plane.

GPU entry points (sm_100a kernels in csrc/lz_codec.cu):
    blob = encode(t)                      # uint8 CUDA tensor, compact stream
    blob = encode(t, level="pack")        # fast level: table codes instead of rANS
    t2 = decode(blob, like=t)             # bit-exact reconstruction
    slots, sizes = encode_slotted(t)      # fixed-capacity per-table-group records
CPU oracle (csrc/cpu/lz_cpu.cpp, bit-identical streams):
    blob = encode_cpu(t); t2 = decode_cpu(blob, n, dtype)

Replaces the reference's external dietgpu codec
(torch.ops.dietgpu.compress_data / decompress_data,
back_up_nccl_allreduce_benchmark/test_dietgpu.py:19-44 of the reference). Unlike
dietgpu, a corrupt stream is reported through a status value, never a device
assert, and the compressed size is measured, not assumed.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from .. import _native, _native_sigs
from ..utils.dtypes import LZ_BF16, LZ_F16, LZ_F32, LZ_U8
from ..utils.trace import traced

c_size, c_ptr, c_int, c_u64, c_u32 = C.c_size_t, C.c_void_p, C.c_int, C.c_uint64, C.c_uint32

_native_sigs.add_cuda({
    "lz_codec_tg_elems": (c_size,),
    "lz_codec_tg_capacity": (c_size, c_int),
    "lz_codec_max_bytes": (c_size, c_size, c_int),
    "lz_codec_scratch_bytes": (c_size, c_size, c_int),
    "lz_codec_encode_slotted": (c_int, c_ptr, c_size, c_int, c_ptr, c_ptr, c_int, c_ptr),
    "lz_codec_decode_slotted": (c_int, c_ptr, c_ptr, c_size, c_int, c_ptr, c_int, c_ptr),
    "lz_codec_encode": (c_int, c_ptr, c_size, c_int, c_ptr, c_size, c_ptr, c_size, c_ptr, c_int, c_ptr),
    "lz_codec_decode": (c_int, c_ptr, c_size, c_ptr, c_size, c_int, c_ptr, c_int, c_ptr),
})
_native_sigs.add_cpu({
    "lzc_tg_capacity": (c_u32, c_u32, c_int),
    "lzc_max_stream_bytes": (c_u64, c_u64, c_int),
    "lzc_tg_encode": (C.c_int64, c_ptr, c_u32, c_int, c_ptr),
    "lzc_tg_decode": (c_int, c_ptr, c_u64, c_ptr, c_u32, c_int),
    "lzc_encode": (C.c_int64, c_ptr, c_u64, c_int, c_ptr, c_u64),
    "lzc_decode": (c_int, c_ptr, c_u64, c_ptr, c_u64, c_int),
    "lzc_histogram": (None, c_ptr, c_u64, c_int, c_ptr),
    "lz_cpu_pack_e4m3": (None, c_ptr, c_ptr, c_u64),
    "lz_cpu_unpack_e4m3": (None, c_ptr, c_ptr, c_u64),
    "lz_cpu_pack_e5m2": (None, c_ptr, c_ptr, c_u64),
    "lz_cpu_unpack_e5m2": (None, c_ptr, c_ptr, c_u64),
})

TG_ELEMS = 32768
LEVELS = {"ans": 0, "pack": 1}  # encoder levels (csrc/lz_codec_format.h)
LEVEL_SHIFT = 8


def level_code(level) -> int:
    """Encoder level name ("ans": rANS, best ratio; "pack": <= 4-bit table
    codes with escapes, a few integer operations per element) or number."""
    if isinstance(level, str):
        if level not in LEVELS:
            raise ValueError(f"unknown codec level {level!r}; expected one of {sorted(LEVELS)}")
        return LEVELS[level]
    if level not in LEVELS.values():
        raise ValueError(f"unknown codec level {level!r}")
    return int(level)


def with_level(dt: int, level) -> int:
    """dtype argument of the native encoders: dtype code | level << 8."""
    return dt | (level_code(level) << LEVEL_SHIFT)


class CodecError(RuntimeError):
    """A compressed stream failed validation."""


def codec_dtype(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return LZ_BF16
    if dtype == torch.float16:
        return LZ_F16
    if dtype == torch.float32:
        return LZ_F32
    if dtype == torch.uint8 or dtype in _fp8_types():
        return LZ_U8
    raise TypeError(f"codec does not support {dtype}")


def _fp8_types():
    return tuple(d for d in (getattr(torch, "float8_e4m3fn", None), getattr(torch, "float8_e5m2", None)) if d)


def _as_bytes_view(t: torch.Tensor) -> torch.Tensor:
    if t.dtype in _fp8_types():
        return t.view(torch.uint8)
    return t


DT_E4M3P, DT_E5M2P = 4, 5
FP8_PAIRS = True  # code fp8 data as packed pairs (one rANS symbol per two values)


def plan(t_dtype: torch.dtype, numel: int):
    """(codec dtype code, codec element count) for a tensor of `numel` values."""
    if t_dtype in _fp8_types() and FP8_PAIRS and numel % 2 == 0:
        return (DT_E4M3P if t_dtype == torch.float8_e4m3fn else DT_E5M2P), numel // 2
    return codec_dtype(t_dtype), numel


def tg_capacity(dtype: torch.dtype) -> int:
    return int(_native.cpu().lzc_tg_capacity(TG_ELEMS, codec_dtype(dtype)))


def max_encoded_bytes(n: int, dtype: torch.dtype) -> int:
    return int(_native.cpu().lzc_max_stream_bytes(n, codec_dtype(dtype)))


# ----------------------------------------------------------------------------- CPU oracle
def encode_cpu(t: torch.Tensor, level="ans") -> torch.Tensor:
    """Compact LZC1 stream of a contiguous CPU tensor (uint8 tensor)."""
    t = t.detach().contiguous().cpu()
    dt, n = plan(t.dtype, t.numel())
    t = _as_bytes_view(t)
    cap = int(_native.cpu().lzc_max_stream_bytes(n, dt))
    out = torch.empty(cap, dtype=torch.uint8)
    rc = _native.cpu().lzc_encode(t.data_ptr(), n, with_level(dt, level), out.data_ptr(), cap)
    if rc < 0:
        raise CodecError(f"lzc_encode failed ({rc})")
    return out[:rc].clone()


def decode_cpu(blob: torch.Tensor, n: int, dtype: torch.dtype) -> torch.Tensor:
    blob = blob.contiguous().cpu()
    dt, ne = plan(dtype, n)
    store = torch.uint8 if dtype in _fp8_types() else dtype
    out = torch.empty(n, dtype=store)
    rc = _native.cpu().lzc_decode(blob.data_ptr(), blob.numel(), out.data_ptr(), ne, dt)
    if rc != 0:
        raise CodecError(f"corrupt LZC1 stream (code {rc})")
    return out.view(dtype) if store != dtype else out


def tg_encode_cpu(t: torch.Tensor, level="ans") -> torch.Tensor:
    """One table-group record (<= 32768 elements)."""
    t = _as_bytes_view(t.detach().contiguous().cpu())
    cap = int(_native.cpu().lzc_tg_capacity(t.numel(), codec_dtype(t.dtype)))
    out = torch.zeros(cap, dtype=torch.uint8)
    rc = _native.cpu().lzc_tg_encode(t.data_ptr(), t.numel(), with_level(codec_dtype(t.dtype), level),
                                     out.data_ptr())
    if rc < 0:
        raise CodecError(f"lzc_tg_encode failed ({rc})")
    return out[:rc].clone()


def tg_decode_cpu(rec: torch.Tensor, n: int, dtype: torch.dtype) -> torch.Tensor:
    rec = rec.contiguous().cpu()
    store = torch.uint8 if dtype in _fp8_types() else dtype
    out = torch.empty(n, dtype=store)
    rc = _native.cpu().lzc_tg_decode(rec.data_ptr(), rec.numel(), out.data_ptr(), n, codec_dtype(dtype))
    if rc != 0:
        raise CodecError(f"corrupt TG record (code {rc})")
    return out.view(dtype) if store != dtype else out


def symbol_entropy_bits(t: torch.Tensor) -> float:
    """Shannon entropy (bits/element) of the symbol plane (order-0, whole tensor)."""
    t = _as_bytes_view(t.detach().contiguous().cpu())
    counts = (C.c_uint64 * 256)()
    _native.cpu().lzc_histogram(t.data_ptr(), t.numel(), codec_dtype(t.dtype), counts)
    n = float(t.numel())
    return -sum((c / n) * math.log2(c / n) for c in counts if c)


# ----------------------------------------------------------------------------- GPU
def _stream_ptr(stream=None) -> int:
    return (stream or torch.cuda.current_stream()).cuda_stream


@traced("encode")
def encode(t: torch.Tensor, nblocks: int = 0, stream=None, return_size: bool = True, level="ans"):
    """Compress a contiguous CUDA tensor into a compact LZC1 stream.

    Returns the stream as a uint8 CUDA tensor trimmed to its size (this reads
    the size back, i.e. synchronises the stream). With ``return_size=False``
    returns ``(buffer, total_bytes_device_tensor)`` without a sync.
    ``level``: "ans" (rANS symbol sections) or "pack" (table codes, faster,
    lower ratio); :func:`decode` reads either.
    """
    if not t.is_cuda:
        return encode_cpu(t, level)
    L = _native.cuda()
    t = t.contiguous()
    dt, n = plan(t.dtype, t.numel())
    t = _as_bytes_view(t)
    cap = L.lz_codec_max_bytes(n, dt)
    scratch = torch.empty(L.lz_codec_scratch_bytes(n, dt), dtype=torch.uint8, device=t.device)
    out = torch.empty(cap, dtype=torch.uint8, device=t.device)
    total = torch.zeros(1, dtype=torch.int64, device=t.device)
    _native.check(L.lz_codec_encode(t.data_ptr(), n, with_level(dt, level), scratch.data_ptr(), scratch.numel(),
                                    out.data_ptr(), cap, total.data_ptr(), nblocks, _stream_ptr(stream)),
                  "lz_codec_encode")
    if not return_size:
        return out, total
    return out[: int(total.item())]


@traced("decode")
def decode(blob: torch.Tensor, like: torch.Tensor | None = None, n: int | None = None,
           dtype: torch.dtype | None = None, out: torch.Tensor | None = None, nblocks: int = 0,
           stream=None, check: bool = True) -> torch.Tensor:
    """Decompress a compact LZC1 stream on the GPU (bit-exact)."""
    if like is not None:
        n, dtype = like.numel(), like.dtype
    if not blob.is_cuda:
        return decode_cpu(blob, n, dtype)
    L = _native.cuda()
    store = torch.uint8 if dtype in _fp8_types() else dtype
    if out is None:
        out = torch.empty(n, dtype=store, device=blob.device)
    status = torch.zeros(1, dtype=torch.int32, device=blob.device)
    dtc, ne = plan(dtype, n)
    _native.check(L.lz_codec_decode(blob.data_ptr(), blob.numel(), out.data_ptr(), ne, dtc,
                                    status.data_ptr(), nblocks, _stream_ptr(stream)), "lz_codec_decode")
    if check:
        st = int(status.item())
        if st:
            raise CodecError(f"corrupt LZC1 stream (status {st})")
    res = out.view(dtype) if store != dtype else out
    return res.view(like.shape) if like is not None else res


def encode_slotted(t: torch.Tensor, nblocks: int = 0, stream=None, level="ans"):
    """Per-table-group records at fixed offsets (t * tg_capacity). Returns (slots, sizes)."""
    L = _native.cuda()
    t = _as_bytes_view(t.contiguous())
    n, dt = t.numel(), codec_dtype(t.dtype)
    ntg = (n + TG_ELEMS - 1) // TG_ELEMS
    cap = L.lz_codec_tg_capacity(dt)
    slots = torch.empty(ntg * cap, dtype=torch.uint8, device=t.device)
    sizes = torch.empty(ntg, dtype=torch.int32, device=t.device)
    _native.check(L.lz_codec_encode_slotted(t.data_ptr(), n, with_level(dt, level), slots.data_ptr(), sizes.data_ptr(),
                                            nblocks, _stream_ptr(stream)), "lz_codec_encode_slotted")
    return slots, sizes


def decode_slotted(slots: torch.Tensor, n: int, dtype: torch.dtype, out: torch.Tensor | None = None,
                   nblocks: int = 0, stream=None, check: bool = True) -> torch.Tensor:
    L = _native.cuda()
    store = torch.uint8 if dtype in _fp8_types() else dtype
    if out is None:
        out = torch.empty(n, dtype=store, device=slots.device)
    status = torch.zeros(1, dtype=torch.int32, device=slots.device)
    _native.check(L.lz_codec_decode_slotted(slots.data_ptr(), out.data_ptr(), n, codec_dtype(dtype),
                                            status.data_ptr(), nblocks, _stream_ptr(stream)),
                  "lz_codec_decode_slotted")
    if check and int(status.item()):
        raise CodecError(f"corrupt table-group record (status {int(status.item())})")
    return out.view(dtype) if store != dtype else out


def compression_ratio(t: torch.Tensor, level="ans") -> float:
    """Measured compressed/raw size of `t` (LZC1 compact stream)."""
    blob = encode(t, level=level) if t.is_cuda else encode_cpu(t, level)
    return blob.numel() / (t.numel() * t.element_size())
