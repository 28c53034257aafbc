"""Per-size algorithm choice for ``allreduce(algo="auto")``.

Thresholds come from bus-bandwidth sweeps on 8xB200 (NVLink 5 / NVSwitch)
with ``python -m results_b200.bench.allreduce_sweep``; the table is keyed by
world size. Until a world size has been measured the defaults below apply:
one-shot for latency-bound messages, NVLS (switch reduction) for large ones
when a multicast object exists, else two-shot.
"""
from __future__ import annotations

KiB = 1 << 10
MiB = 1 << 20

# world -> list of (max_bytes, algo_with_multicast, algo_without_multicast).
# 2 GPUs (sweep of 2xB200, bf16): one-shot wins up to 8 MB, two-shot above
# (NVLS moves (1 + 1/N) S per GPU but is slower than two-shot's S at N = 2).
# 8 GPUs: NVLS wins from 64 MB (621 vs 517 two-shot, NCCL 421) to 1 GB
# (809 vs 646, NCCL 725).
# Low-latency one-shot (flag-in-data pushes, no barrier) below 256 KB: 2xB200,
# CUDA-graph device time, 1 KB 3.9 us and 256 KB 6.2 us vs NCCL 14.6 / 18.4 us.
TABLE = {
    2: [
        (256 * 1024, "ll", "ll"),
        (8 * MiB, "oneshot", "oneshot"),
        (1 << 62, "twoshot", "twoshot"),
    ],
    "default": [
        (256 * 1024, "ll", "ll"),
        (4 * MiB, "oneshot", "oneshot"),
        (1 << 62, "nvls", "twoshot"),
    ],
}


def choose(nbytes: int, world: int, has_multicast: bool, symmetric: bool) -> str:
    rows = TABLE.get(world, TABLE["default"])
    for max_b, with_mc, without_mc in rows:
        if nbytes <= max_b:
            algo = with_mc if has_multicast else without_mc
            if nbytes % 16 and algo != "oneshot":
                return "oneshot" if nbytes <= 4 * MiB else "twoshot"
            return algo
    return "twoshot"
