"""SM budgets through CUDA green contexts.

    with SmBudget(device=0, sm_count=16) as b:
        with torch.cuda.stream(b.stream):
            lz.compressed_allreduce(x)      # runs on at most b.sm_count SMs

The B200 counterpart of back_up/green_context_example.cu:15-79 and of the
UCCL engine's green-context SM partitions (16/32/64/100 of 132 SMs on H200;
on B200's 148 SMs the sweep uses 16/32/64/96/128). ``probe_smids`` launches
blocks that record ``%smid`` so a budget can be checked.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _native, _native_sigs

_native_sigs.add_cuda({
    "lz_sm_budget_create": (C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                            C.POINTER(C.c_int)),
    "lz_sm_budget_destroy": (C.c_int, C.c_void_p),
    "lz_smid_probe": (C.c_int, C.c_void_p, C.c_void_p, C.c_int),
})

SWEEP = (16, 32, 64, 96, 128)


class SmBudget:
    def __init__(self, device: int | None = None, sm_count: int = 16):
        self.device = torch.cuda.current_device() if device is None else device
        self._lib = _native.cuda()
        self._h = C.c_void_p()
        raw = C.c_void_p()
        granted = C.c_int()
        _native.check(self._lib.lz_sm_budget_create(self.device, sm_count, C.byref(self._h), C.byref(raw),
                                                    C.byref(granted)), "sm budget")
        self.sm_count = granted.value
        self.stream = torch.cuda.ExternalStream(raw.value, device=torch.device("cuda", self.device))

    def close(self):
        if self._h:
            self._lib.lz_sm_budget_destroy(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def probe_smids(stream: torch.cuda.Stream, nblocks: int = 256) -> list[int]:
    """SM id of every block of a probe launch on `stream`."""
    out = torch.full((nblocks,), -1, dtype=torch.int32, device=stream.device)
    _native.check(_native.cuda().lz_smid_probe(stream.cuda_stream, out.data_ptr(), nblocks), "smid probe")
    stream.synchronize()
    return out.tolist()
