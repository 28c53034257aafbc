"""dtype codes shared with the native library (enum LzDtype in csrc/lz_types.h)."""
from __future__ import annotations

import torch

LZ_F32, LZ_F16, LZ_BF16, LZ_U8 = 0, 1, 2, 3

_MAP = {
    torch.float32: LZ_F32,
    torch.float16: LZ_F16,
    torch.bfloat16: LZ_BF16,
    torch.uint8: LZ_U8,
}


def lz_dtype(dt: torch.dtype) -> int:
    try:
        return _MAP[dt]
    except KeyError:
        raise TypeError(f"dtype {dt} is not supported by the native kernels") from None


FP8_DTYPES = tuple(d for d in (getattr(torch, "float8_e4m3fn", None), getattr(torch, "float8_e5m2", None)) if d is not None)
