"""Public allreduce entry point with per-size algorithm selection.

``allreduce(t, algo=...)`` covers every variant of the reference's
benchmark driver (single_node_nccl_allreduce_benchmark/benchmark_both.py:372-383,
16_node_nccl_allreduce_benchmark/benchmark_both.py:156-176):

* native sm_100a kernels over NVLink peer memory / NVLS (CUDA tensors):
  ``oneshot``, ``twoshot`` (alias ``p2p``), ``nvls``, ``nvls_oneshot``,
  ``ring`` (alias ``ringp2p``), ``rhd``, ``ll`` (low-latency one-shot,
  flag-in-data pushes, messages up to 256 KB);
* ``ce`` (alias ``memcpy``): copy-engine two-shot, bytes moved by DMA and
  reduced by a kernel (zero-copy and pipelined for symmetric, distinct
  input and output);
* NCCL baseline: ``nccl`` (``dist.all_reduce``);
* host-orchestrated send/recv reference algorithms (any backend, also CPU):
  ``naive``, ``naive_twoshot``, ``ring_sendrecv``, ``rhd_sendrecv``,
  ``twoshot_collective``, ``multichannel_ring``, ``hierarchical``;
* ``auto``: the measured size table of :mod:`results_b200.parallel.tuning`.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..config import Config
from ..utils.trace import traced
from .comm import Communicator

_DEFAULT: Communicator | None = None

NATIVE = {"oneshot", "twoshot", "nvls", "nvls_oneshot", "ring", "rhd", "ll", "ce"}
ALIASES = {"p2p": "twoshot", "ringp2p": "ring", "two_shot": "twoshot", "one_shot": "oneshot", "memcpy": "ce"}
HOST_ALGOS = {"naive", "naive_twoshot", "ring_sendrecv", "rhd_sendrecv", "twoshot_collective",
              "multichannel_ring", "hierarchical", "pipelined_twoshot"}


def init(group=None, config: Config | None = None) -> Communicator:
    """Create (collectively) the default communicator for ``group``."""
    global _DEFAULT
    if _DEFAULT is None:
        _DEFAULT = Communicator(group=group, config=config)
    return _DEFAULT


def get_comm() -> Communicator | None:
    return _DEFAULT


def shutdown() -> None:
    global _DEFAULT
    if _DEFAULT is not None:
        _DEFAULT.close()
        _DEFAULT = None


def select_algo(nbytes: int, world: int, has_multicast: bool, symmetric: bool,
                config: Config | None = None, out_of_place: bool = True) -> str:
    """Algorithm for a message: ``config.algo`` when it names one, else the
    measured size table (``symmetric``: input and output in the heap;
    ``out_of_place``: they are distinct buffers)."""
    from .tuning import choose

    if config is not None and config.algo not in ("", "auto"):
        return ALIASES.get(config.algo, config.algo)
    return choose(nbytes, world, has_multicast, symmetric, out_of_place,
                  exact=bool(config is not None and config.exact))


def _padded_allreduce(comm, t: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    """Large tensor whose size or address is not a multiple of 16 bytes: the
    vector kernels run on a zero-padded aligned copy (zeros add nothing to the
    sum), and the result is copied back. The padded buffer is kept on the
    communicator and only grows, so repeated calls do not allocate."""
    es = t.element_size()
    n = t.numel()
    need = (n + (-(n * es) % 16) // es) * es
    buf = getattr(comm, "_pad_scratch", None)
    if buf is None or buf.numel() < need:
        buf = torch.empty(need, dtype=torch.uint8, device=t.device)
        comm._pad_scratch = buf
    tmp = buf[:need].view(t.dtype)
    tmp[n:].zero_()
    tmp[:n].copy_(t.reshape(-1))
    comm.allreduce_(tmp, algo="twoshot")
    res = t if out is None else out
    res.copy_(tmp[:n].view(t.shape))
    return res


@traced("allreduce")
def allreduce(t: torch.Tensor, algo: str = "auto", out: torch.Tensor | None = None,
              comm: Communicator | None = None, group=None) -> torch.Tensor:
    """Sum-allreduce ``t`` across the group. In place unless ``out`` is given."""
    algo = ALIASES.get(algo, algo)
    if algo == "nccl" or (not t.is_cuda and algo in ("auto", "nccl")):
        res = t if out is None else out.copy_(t)
        dist.all_reduce(res, op=dist.ReduceOp.SUM, group=group)
        return res
    if algo in HOST_ALGOS:
        from . import sendrecv

        res = t if out is None else out.copy_(t)
        sendrecv.allreduce(res, algo, group=group)
        return res
    comm = comm or _DEFAULT or init(group)
    if algo == "auto":
        out_of_place = out is not None and out.data_ptr() != t.data_ptr()
        algo = select_algo(t.numel() * t.element_size(), comm.world, comm.has_multicast,
                           comm.is_symmetric(t) and (out is None or comm.is_symmetric(out)),
                           comm.config, out_of_place)
        nbytes = t.numel() * t.element_size()
        if algo != "oneshot" and (nbytes % 16 or t.data_ptr() % 16 or (out is not None and out.data_ptr() % 16)):
            if nbytes <= comm.config.oneshot_bytes:
                algo = "oneshot"
            else:
                return _padded_allreduce(comm, t, out)
    if algo not in NATIVE:
        raise ValueError(f"unknown allreduce algorithm {algo!r}")
    return comm.allreduce_(t, out, algo=algo)
