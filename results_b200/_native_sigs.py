"""ctypes signatures of the native subsystems (declared when the symbol exists)."""
from __future__ import annotations

import ctypes as C

c_size = C.c_size_t
c_ptr = C.c_void_p
c_int = C.c_int
c_dbl = C.c_double
c_u64 = C.c_uint64
c_u32 = C.c_uint32
P = C.POINTER

_CUDA = {
    # single-GPU emulation
    "lz_emu_create": (c_int, c_int, c_size, c_size, c_size, c_dbl, P(c_ptr)),
    "lz_emu_destroy": (c_int, c_ptr),
    "lz_emu_heap_ptr": (c_ptr, c_ptr, c_int),
    "lz_emu_user_offset": (c_size, c_ptr),
    "lz_emu_status": (c_int, c_ptr, c_int),
    "lz_emu_allreduce": (c_int, c_ptr, P(c_ptr), P(c_ptr), c_size, c_int, c_int, c_int, c_int, c_ptr),
}

_CUDA["lz_test_wait_timeout"] = (c_int, c_ptr, c_dbl, c_ptr)
# copy-engine allreduce (csrc/lz_copy_engine.cu)
_CUDA["lz_ce_allreduce"] = (c_int, c_ptr, c_ptr, c_ptr, c_size, c_int, c_int, c_ptr)
_CUDA["lz_ce_allreduce_is_zero_copy"] = (c_int, c_ptr, c_ptr, c_ptr, c_size, c_int)
_CUDA["lz_emu_weight_transfer"] = (c_int, c_ptr, c_int, c_u32, P(c_ptr), c_u32, c_int, c_int, c_int,
                                   P(c_u64), c_ptr)

_CPU = {}


_LOADED = {"cuda": None, "cpu": None}


def _apply(lib, table, sig) -> None:
    for name, (res, *args) in table.items():
        if hasattr(lib, name):
            sig(lib, name, res, *args)


def declare(lib, sig) -> None:
    _LOADED["cuda"] = (lib, sig)
    _apply(lib, _CUDA, sig)


def declare_cpu(lib, sig) -> None:
    _LOADED["cpu"] = (lib, sig)
    _apply(lib, _CPU, sig)


def add_cuda(table: dict) -> None:
    """Register signatures; applied now if the library is already loaded."""
    _CUDA.update(table)
    if _LOADED["cuda"] is not None:
        _apply(_LOADED["cuda"][0], table, _LOADED["cuda"][1])


def add_cpu(table: dict) -> None:
    _CPU.update(table)
    if _LOADED["cpu"] is not None:
        _apply(_LOADED["cpu"][0], table, _LOADED["cpu"][1])
