"""Library configuration.

One frozen dataclass, populated from ``LZ_*`` environment variables and
overridable per call with :func:`dataclasses.replace`. It replaces the
scattered knobs of the reference: ``RING_NUM_CHANNELS`` / ``HD_MAX_MB``
(16_node_nccl_allreduce_benchmark/ring_sendrecv_allreduce.py:33-36), the
``COMP_RATIO`` constants (single_node_nccl_allreduce_benchmark/compressed_twoshot_allreduce.py:49,
single_node_nccl_allreduce_benchmark/compressed_p2p_allreduce.py:51), the 16 M-element pipeline
threshold (16_node_nccl_allreduce_benchmark/naive_sendrecv_allreduce.py:40) and the
``update_weight_buffer_size`` argument of the weight updater
(back_up/update_weight_from_distributed.py:259).
"""
from __future__ import annotations

import dataclasses
import os

MiB = 1 << 20
GiB = 1 << 30


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def _env_float(name: str, default: float) -> float:
    v = os.environ.get(name)
    return float(v) if v not in (None, "") else default


def _env_str(name: str, default: str) -> str:
    v = os.environ.get(name)
    return v if v not in (None, "") else default


def _env_bool(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    if v in (None, ""):
        return default
    return v.lower() not in ("0", "false", "no", "off")


@dataclasses.dataclass(frozen=True)
class Config:
    # symmetric heap layout (bytes per rank)
    heap_bytes: int = 0               # 0: oneshot*2 + stage + user_bytes
    user_bytes: int = 1 * GiB         # region for symmetric (zero-copy) tensors
    oneshot_bytes: int = 8 * MiB      # largest one-shot message (double buffered)
    stage_bytes: int = 1 * GiB        # staging for non-symmetric two-shot / NVLS / ring / RHD
    use_multicast: bool = True        # bind an NVLS multicast object when supported
    # device waits
    timeout_s: float = 10.0
    # launch shape
    nthreads: int = 0                 # 0: per-algorithm launch shape measured on B200
    sm_budget: int = 0                # 0: all SMs; otherwise the grid is capped to this
    # algorithm selection (bytes); measured on 8xB200, see results_b200/parallel/tuning.py
    algo: str = "auto"
    exact: bool = False               # auto picks only bit-exact algorithms (never NVLS)
    # ring / halving-doubling channel knobs of the send/recv reference suite
    ring_channels: int = 4
    hd_max_bytes: int = 128 * MiB
    pipeline_min_elements: int = 16 * 1024 * 1024
    # codec
    codec: str = "split_ans"          # "raw" | "split_ans"
    ratio_budget: float = 0.65        # fixed-size budget of the host compressed ring / two-shot messages
    chunk_bytes: int = 64 * MiB       # pipelining unit of weight transfer / compressed paths
    # weight transfer
    update_weight_buffer_bytes: int = 512 * MiB

    @staticmethod
    def from_env() -> "Config":
        d = Config()
        return dataclasses.replace(
            d,
            heap_bytes=_env_int("LZ_HEAP_BYTES", d.heap_bytes),
            user_bytes=_env_int("LZ_USER_BYTES", d.user_bytes),
            oneshot_bytes=_env_int("LZ_ONESHOT_BYTES", d.oneshot_bytes),
            stage_bytes=_env_int("LZ_STAGE_BYTES", d.stage_bytes),
            use_multicast=_env_bool("LZ_MULTICAST", d.use_multicast),
            timeout_s=_env_float("LZ_TIMEOUT_S", d.timeout_s),
            nthreads=_env_int("LZ_NTHREADS", d.nthreads),
            sm_budget=_env_int("LZ_SM_BUDGET", d.sm_budget),
            algo=_env_str("LZ_ALGO", d.algo),
            exact=_env_bool("LZ_EXACT", d.exact),
            ring_channels=_env_int("RING_NUM_CHANNELS", _env_int("LZ_RING_CHANNELS", d.ring_channels)),
            hd_max_bytes=_env_int("HD_MAX_MB", d.hd_max_bytes // MiB) * MiB,
            pipeline_min_elements=_env_int("LZ_PIPELINE_MIN_ELEMENTS", d.pipeline_min_elements),
            codec=_env_str("LZ_CODEC", d.codec),
            ratio_budget=_env_float("LZ_RATIO_BUDGET", d.ratio_budget),
            chunk_bytes=_env_int("LZ_CHUNK_BYTES", d.chunk_bytes),
            update_weight_buffer_bytes=_env_int("LZ_UPDATE_WEIGHT_BUFFER_BYTES",
                                                d.update_weight_buffer_bytes),
        )

    def total_heap_bytes(self) -> int:
        if self.heap_bytes:
            return self.heap_bytes
        # flags (1 MiB) + one-shot double buffer + low-latency areas (2 parities x
        # up to 8 ranks x 2 x 256 KB = 8 MiB) + stage + user + alignment slack
        return (1 * MiB) + 2 * self.oneshot_bytes + 8 * MiB + self.stage_bytes + self.user_bytes + 4 * MiB
