"""Tracing: NVTX ranges around every host-visible phase, and log lines.

Every public entry point (allreduce, compressed_allreduce, all_to_all,
weight send / recv / broadcast per bucket, codec encode / decode, fp8 pack /
unpack, the host-orchestrated compressed variants' compress / exchange /
decompress steps) opens an NVTX range named ``lz:<what>`` when tracing is on,
so an nsys or ncu timeline shows where each call's kernels belong. Inside a
persistent kernel the phases are separated by device barriers and are not
visible to NVTX; their cost is measured with the kernels' profiling hooks
(e.g. ``LZ_CODEC_STOP_AFTER``) instead.

Enable with ``LZ_NVTX=1`` (read once) or :func:`enable`. The reference has only
CUDA-event timing and the UCCL engine's ``split=..us, encode=..us`` log lines
(its raw/bf16_split_sm16_split_encode_time_count.txt); the weight updater's
bucket log lines are emitted through :data:`log` at INFO level.
"""
from __future__ import annotations

import contextlib
import functools
import logging
import os

log = logging.getLogger("results_b200")

_ENABLED = os.environ.get("LZ_NVTX", "0") not in ("", "0")


def enable(on: bool = True) -> None:
    global _ENABLED
    _ENABLED = bool(on)


def enabled() -> bool:
    return _ENABLED


@contextlib.contextmanager
def range(name: str):  # noqa: A001 - mirrors nvtx.range
    """NVTX range ``lz:<name>`` while tracing is enabled; a no-op otherwise."""
    if not _ENABLED:
        yield
        return
    import torch

    torch.cuda.nvtx.range_push(f"lz:{name}")
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def traced(name: str):
    """Decorator form of :func:`range` (the range carries the ``algo`` kwarg when given)."""

    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            if not _ENABLED:
                return fn(*args, **kwargs)
            algo = kwargs.get("algo")
            with range(f"{name}[{algo}]" if algo else name):
                return fn(*args, **kwargs)

        return wrapper

    return deco
