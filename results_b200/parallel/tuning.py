"""Per-size algorithm choice for ``allreduce(algo="auto")``.

Thresholds come from bus-bandwidth sweeps on 8xB200 (NVLink 5 / NVSwitch)
with ``python -m results_b200.bench.allreduce_sweep``; the table is keyed by
world size. Until a world size has been measured the defaults below apply:
one-shot for latency-bound messages, NVLS (switch reduction) for large ones
when a multicast object exists, else two-shot.

The reference picks by size too, with fixed thresholds: halving-doubling up
to HD_MAX_MB and K-channel rings by size
(16_node_nccl_allreduce_benchmark/ring_sendrecv_allreduce.py:33-36,254-313),
and a fused all-source reduce below 1 M elements
(single_node_nccl_allreduce_benchmark/compressed_p2p_kernel.cu:304-305).
"""
from __future__ import annotations

KiB = 1 << 10
MiB = 1 << 20

# world -> list of (max_bytes, algo_with_multicast, algo_without_multicast).
# Rows: (largest message in bytes, algorithm with NVLS multicast, without).
# Fitted to CUDA-graph device times of the bf16 sweep on B200
# (bench/allreduce_sweep.py --graph, max over ranks):
#   2 GPUs: ll 3.9 us at 1 KB .. 6.2 us at 256 KB (NCCL 14.6 .. 18.4); one-shot
#           up to 8 MB; two-shot kernel up to 128 MB; copy-engine two-shot
#           ("ce", symmetric out-of-place buffers) from 256 MB (256 MB: 650 vs
#           two-shot 592 GB/s busbw; 1 GB: 741 vs 596, NCCL 565). NVLS moves
#           (1 + 1/N) S per GPU, more than two-shot's S at N = 2.
#   4 GPUs: ll to 256 KB; one-shot to 2 MB; two-shot 4 MB .. 256 MB; NVLS at
#           512 MB (672 vs two-shot 642 GB/s busbw); copy-engine two-shot from
#           1 GB (689, bit-exact, vs NVLS 685 and NCCL 642).
# NVLS reduces inside the switch: measured within 1 ulp of the fp32 rank-order
# sum up to 512 MB and 2-4 ulp at 1 GB (rare near-cancelling elements); with
# exact=True (Config.exact, LZ_EXACT=1) the table never picks it and the
# bit-exact copy-engine or two-shot path takes its rows.
#   8 GPUs: ll to 128 KB; one-shot to 512 KB; two-shot 1 .. 8 MB; NVLS from
#           16 MB (1 GB: 2329 us vs NCCL 2595, 64 MB: 190 vs 278).
TABLE = {
    2: [
        (256 * 1024, "ll", "ll"),
        (8 * MiB, "oneshot", "oneshot"),
        (128 * MiB, "twoshot", "twoshot"),
        (1 << 62, "ce", "ce"),
    ],
    4: [
        (256 * 1024, "ll", "ll"),
        (2 * MiB, "oneshot", "oneshot"),
        (256 * MiB, "twoshot", "twoshot"),
        (512 * MiB, "nvls", "twoshot"),
        (1 << 62, "ce", "ce"),
    ],
    8: [
        (128 * 1024, "ll", "ll"),
        (512 * 1024, "oneshot", "oneshot"),
        (8 * MiB, "twoshot", "twoshot"),
        (1 << 62, "nvls", "twoshot"),
    ],
    "default": [
        (128 * 1024, "ll", "ll"),
        (1 * MiB, "oneshot", "oneshot"),
        (1 << 62, "nvls", "twoshot"),
    ],
}


def choose(nbytes: int, world: int, has_multicast: bool, symmetric: bool, out_of_place: bool = True,
           exact: bool = False) -> str:
    """Row of TABLE for (world, nbytes). The copy-engine two-shot ("ce") is
    zero-copy only for symmetric, distinct input and output; otherwise the
    two-shot kernel takes its rows. ``exact``: only algorithms whose result is
    bit-identical to the fp32 rank-order sum (no NVLS)."""
    rows = TABLE.get(world, TABLE["default"])
    for max_b, with_mc, without_mc in rows:
        if nbytes <= max_b:
            algo = with_mc if has_multicast else without_mc
            if exact and algo.startswith("nvls"):
                algo = "ce" if nbytes >= 256 * MiB else "twoshot"
            if algo == "ce" and not (symmetric and out_of_place and nbytes % (16 * world) == 0):
                algo = "twoshot"
            if nbytes % 16 and algo != "oneshot":
                return "oneshot" if nbytes <= 4 * MiB else "twoshot"
            return algo
    return "twoshot"
