"""Compression-ratio log parsers.

Counterparts of raw/avg_compression_ratio.py:1-23 and
raw/avg_compression_ratio_by_weight.py:1-36 of the reference, which average the
ratios printed by the UCCL engine (``... Compressed X bytes to Y bytes,
ratio R``) per message size or per weight name. The same line format is
accepted here, plus this library's own ``codec: name=... raw=X comp=Y`` lines.

    python -m results_b200.utils.logparse by-size  run.log
    python -m results_b200.utils.logparse by-weight run.log
"""
from __future__ import annotations

import re
import sys
from collections import OrderedDict

_UCCL = re.compile(r"Compressed\s+(\d+)\s+bytes\s+to\s+(\d+)\s+bytes(?:,\s*ratio\s*([0-9.]+))?")
_OURS = re.compile(r"codec:\s*(?:name=(\S+)\s+)?raw=(\d+)\s+comp=(\d+)")
_NAME = re.compile(r"(?:weight|name|tensor)[=:\s]+([A-Za-z0-9_.]+)")


def _records(lines):
    for line in lines:
        m = _UCCL.search(line)
        if m:
            raw, comp = int(m.group(1)), int(m.group(2))
            name = _NAME.search(line)
            yield (name.group(1) if name else None), raw, comp
            continue
        m = _OURS.search(line)
        if m:
            yield m.group(1), int(m.group(2)), int(m.group(3))


def by_size(lines) -> "OrderedDict[int, float]":
    """Average compressed/raw ratio per raw size (first-seen order)."""
    acc: "OrderedDict[int, list]" = OrderedDict()
    for _, raw, comp in _records(lines):
        acc.setdefault(raw, []).append(comp / raw if raw else 0.0)
    return OrderedDict((k, sum(v) / len(v)) for k, v in acc.items())


def by_weight(lines) -> "OrderedDict[str, float]":
    """Average ratio per weight name (lines without a name are grouped by size)."""
    acc: "OrderedDict[str, list]" = OrderedDict()
    for name, raw, comp in _records(lines):
        key = name if name else f"size={raw}"
        acc.setdefault(key, []).append(comp / raw if raw else 0.0)
    return OrderedDict((k, sum(v) / len(v)) for k, v in acc.items())


def log_line(name: str, raw: int, comp: int) -> str:
    """The line format this library emits for every compressed transfer."""
    return f"codec: name={name} raw={raw} comp={comp} ratio={comp / raw if raw else 0:.6f}"


def main(argv=None):
    argv = argv or sys.argv[1:]
    mode, path = argv[0], argv[1]
    with open(path, errors="replace") as f:
        res = (by_size if mode == "by-size" else by_weight)(f)
    for k, v in res.items():
        print(f"{k}\t{v:.6f}")


if __name__ == "__main__":
    main()
