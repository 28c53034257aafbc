"""Register, spill and shared-memory figures of every kernel, from ptxas.

    python -m results_b200.utils.ptxas_report [csrc/lz_allreduce.cu ...]

Compiles each translation unit for sm_100a with ``-Xptxas -v`` (the flags of
:mod:`results_b200.utils.build`) and prints one line per kernel entry:
demangled name, registers per thread, spill stores/loads and static shared
memory. Only what ptxas prints is used.
"""
from __future__ import annotations

import re
import subprocess
import sys
import tempfile
from pathlib import Path

from .build import CSRC, NVCC, NVCC_FLAGS

_ENTRY = re.compile(r"Compiling entry function '(\S+)'")
_SPILL = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")
_USED = re.compile(r"Used (\d+) registers.*?(\d+) bytes smem")


def _demangle(names: list[str]) -> list[str]:
    try:
        out = subprocess.run(["c++filt"], input="\n".join(names), capture_output=True, text=True).stdout
        return out.strip().splitlines()
    except OSError:
        return names


def kernels(src: Path) -> list[dict]:
    with tempfile.TemporaryDirectory() as d:
        cmd = [NVCC, *NVCC_FLAGS, "-diag-suppress=550", "-Xptxas", "-v", "-I", str(CSRC), "-c", str(src),
               "-o", str(Path(d) / "k.o")]
        txt = subprocess.run(cmd, capture_output=True, text=True).stderr
    rows, cur = [], None
    for line in txt.splitlines():
        m = _ENTRY.search(line)
        if m:
            cur = {"mangled": m.group(1), "stack": 0, "spill_st": 0, "spill_ld": 0}
            continue
        m = _SPILL.search(line)
        if m and cur is not None:
            cur["stack"], cur["spill_st"], cur["spill_ld"] = map(int, m.groups())
            continue
        m = _USED.search(line)
        if m and cur is not None:
            cur["regs"], cur["smem"] = int(m.group(1)), int(m.group(2))
            rows.append(cur)
            cur = None
    for r, name in zip(rows, _demangle([r["mangled"] for r in rows])):
        r["name"] = re.sub(r"\(anonymous namespace\)::", "", name)
    return rows


def main(argv=None) -> int:
    srcs = [Path(a) for a in (argv or sys.argv[1:])] or sorted(CSRC.glob("*.cu"))
    for src in srcs:
        print(f"== {src.name}")
        for r in kernels(src):
            print(f"  {r['regs']:4d} regs  spill {r['spill_st']:3d}/{r['spill_ld']:3d} B  smem {r['smem']:6d} B  "
                  f"{r['name'][:150]}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
