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

# world -> list of (max_bytes, algo_with_multicast, algo_without_multicast)
TABLE = {
    "default": [
        (256 * KiB, "oneshot", "oneshot"),
        (1 << 62, "nvls", "twoshot"),
    ],
}


def choose(nbytes: int, world: int, has_multicast: bool, symmetric: bool) -> str:
    rows = TABLE.get(world, TABLE["default"])
    for max_b, with_mc, without_mc in rows:
        if nbytes <= max_b:
            algo = with_mc if has_multicast else without_mc
            if nbytes % 16 and algo != "oneshot":
                return "oneshot" if nbytes <= 8 * MiB else "twoshot"
            return algo
    return "twoshot"
