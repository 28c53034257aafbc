"""ctypes bindings to the in-tree native libraries.

``cuda()`` returns the sm_100a runtime (``liblz_cuda.so``); ``cpu()`` returns the
CPU oracle (``liblz_cpu.so``). Both are built in-tree by
:mod:`results_b200.utils.build`; when a library is missing it is built on first
use, and if that fails on a machine with a GPU the error is raised -- GPU code
paths never fall back silently to PyTorch.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

_LIB_DIR = Path(__file__).resolve().parent / "lib"
_lock = threading.Lock()
_cuda_lib = None
_cpu_lib = None

c_size = C.c_size_t
c_ptr = C.c_void_p
c_int = C.c_int
c_dbl = C.c_double
c_u64 = C.c_uint64
c_u32 = C.c_uint32


class NativeError(RuntimeError):
    """A native call returned an error code."""


class CollectiveTimeout(NativeError):
    """A device-side flag wait expired; the communicator is poisoned."""


def _load(name: str, builder):
    path = _LIB_DIR / name
    if not path.exists() or os.environ.get("LZ_ALWAYS_BUILD"):
        builder()
    return C.CDLL(str(path), mode=C.RTLD_GLOBAL)


def _sig(lib, name, restype, *argtypes):
    f = getattr(lib, name)
    f.restype = restype
    f.argtypes = list(argtypes)
    return f


def cuda():
    """The CUDA runtime library (loaded once)."""
    global _cuda_lib
    if _cuda_lib is not None:
        return _cuda_lib
    with _lock:
        if _cuda_lib is None:
            from .utils import build

            lib = _load(build.cuda_lib_name(), build.build_cuda)
            _declare_cuda(lib)
            _cuda_lib = lib
    return _cuda_lib


def cpu():
    """The CPU oracle library (loaded once)."""
    global _cpu_lib
    if _cpu_lib is not None:
        return _cpu_lib
    with _lock:
        if _cpu_lib is None:
            from .utils import build

            lib = _load("liblz_cpu.so", build.build_cpu)
            _declare_cpu(lib)
            _cpu_lib = lib
    return _cpu_lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = cuda().lz_last_error().decode(errors="replace")
        raise NativeError(f"{what or 'native call'} failed ({rc}): {msg}")


def _declare_cuda(L) -> None:
    P = C.POINTER
    _sig(L, "lz_last_error", C.c_char_p)
    _sig(L, "lz_version", c_int)
    _sig(L, "lz_device_info", c_int, c_int, P(c_int), P(c_int), P(c_int), P(c_int), P(c_size))
    _sig(L, "lz_can_access_peer", c_int, c_int, c_int, P(c_int))
    _sig(L, "lz_nvlink_p2p_attr", c_int, c_int, c_int, P(c_int), P(c_int))
    _sig(L, "lz_heap_create", c_int, c_int, c_int, c_int, c_size, c_int, C.c_char_p, P(c_ptr))
    for n in ("lz_heap_serve", "lz_heap_connect", "lz_mc_create", "lz_mc_attach", "lz_mc_bind",
              "lz_mc_map", "lz_heap_stop_serving", "lz_heap_destroy", "lz_heap_has_mc"):
        _sig(L, n, c_int, c_ptr)
    _sig(L, "lz_heap_size", c_size, c_ptr)
    _sig(L, "lz_heap_ptr", c_ptr, c_ptr, c_int)
    _sig(L, "lz_heap_mc_ptr", c_ptr, c_ptr)
    _sig(L, "lz_comm_create", c_int, c_ptr, c_size, c_size, c_dbl, P(c_ptr))
    _sig(L, "lz_comm_destroy", c_int, c_ptr)
    _sig(L, "lz_comm_user_offset", c_size, c_ptr)
    _sig(L, "lz_comm_status", c_int, c_ptr)
    _sig(L, "lz_comm_clear_status", c_int, c_ptr)
    _sig(L, "lz_comm_epoch", c_int, c_ptr, P(c_u64), c_ptr)
    _sig(L, "lz_allreduce", c_int, c_ptr, c_ptr, c_ptr, c_size, c_int, c_int, c_int, c_int, c_ptr)
    _sig(L, "lz_barrier", c_int, c_ptr, c_ptr)
    _declare_optional_cuda(L)


def _declare_optional_cuda(L) -> None:
    """Symbols of later subsystems; declared when present in the build."""
    from . import _native_sigs

    _native_sigs.declare(L, _sig)


def _declare_cpu(L) -> None:
    from . import _native_sigs

    _native_sigs.declare_cpu(L, _sig)


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def loaded_libraries() -> list[str]:
    out = []
    if _cuda_lib is not None:
        out.append(str(_LIB_DIR / "liblz_cuda.so"))
    if _cpu_lib is not None:
        out.append(str(_LIB_DIR / "liblz_cpu.so"))
    return out
