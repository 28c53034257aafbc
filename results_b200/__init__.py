"""results_b200 -- a Blackwell-native (sm_100a) compressed-collective library.

Public API (the capabilities of the monopodium/results research code,
re-designed for 8xB200 with NVLink 5 / NVSwitch):

* ``init(group, config)`` -> :class:`Communicator` (symmetric heap + NVLS)
* ``allreduce(t, algo="auto")`` -- one-shot, two-shot, NVLS, ring, RHD native
  kernels; NCCL baseline; send/recv reference algorithms
* ``compressed_allreduce(t)`` -- lossless split+rANS compressed two-shot
* ``all_to_all(x, compress=False)`` -- raw or split+rANS compressed all-to-all
* ``send_weights`` / ``recv_weights`` / ``broadcast_weights`` -- RL weight
  update transfer (raw / split+rANS), chunk-pipelined
* ``encode`` / ``decode`` -- the LZC1 lossless float codec
* ``pack_fp8`` / ``unpack_fp8`` -- e4m3 / e5m2 pair packing
"""
from __future__ import annotations

__version__ = "0.1.0"

from .config import Config  # noqa: F401


__all__ = ["Config", "Communicator", "init", "allreduce", "get_comm", "shutdown", "select_algo",
           "compressed_allreduce", "all_to_all", "send_weights", "recv_weights", "broadcast_weights",
           "WeightTransfer", "encode", "decode", "pack_fp8", "unpack_fp8"]


def __dir__():
    return sorted(set(globals()) | set(__all__))


def __getattr__(name):
    # Lazy imports keep `import results_b200` cheap and CPU-safe.
    if name in ("init", "allreduce", "get_comm", "shutdown", "select_algo"):
        from .parallel import allreduce as _ar

        return getattr(_ar, name)
    if name == "Communicator":
        from .parallel.comm import Communicator

        return Communicator
    if name in ("compressed_allreduce",):
        from .parallel import compressed

        return getattr(compressed, name)
    if name in ("all_to_all",):
        from .parallel import alltoall

        return getattr(alltoall, name)
    if name in ("send_weights", "recv_weights", "broadcast_weights", "WeightTransfer"):
        from .parallel import weights

        return getattr(weights, name)
    if name in ("encode", "decode"):
        from .ops import codec

        return getattr(codec, name)
    if name in ("pack_fp8", "unpack_fp8"):
        from .ops import fp8

        return getattr(fp8, name)
    raise AttributeError(name)
