"""Launcher: one process per GPU through torchrun.

    python -m results_b200.launch local 8 -m results_b200.bench.allreduce_sweep --csv out.csv
    python -m results_b200.launch node --nnodes 2 --node-rank 0 --master-addr 10.0.0.1 8 bench.py ...

``local`` runs N ranks on this node (127.0.0.1 rendezvous); ``node`` is the
multi-node form. Counterpart of single_node_nccl_allreduce_benchmark/run.sh:21-44
(``run.sh local`` -> 2 local GPUs, otherwise a 2-node torchrun). Every
launch is bounded by ``timeout -k 60`` well above the process-group
timeout so ranks that wait on each other end with an error.

``--gdbserver PORT`` starts rank 0 under ``gdbserver :PORT`` (the other ranks
run normally), the counterpart of back_up/mpi_gdbserver.sh:1-48: attach a
debugger to the first rank while the job runs.
"""
from __future__ import annotations

import argparse
import os
import shlex
import shutil
import socket
import subprocess
import sys


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# rank 0 under gdbserver, the others as usual ("$@" = python arguments)
_GDB_WRAPPER = ('if [ "$RANK" = "0" ]; then exec gdbserver ":$LZ_GDB_PORT" "$LZ_PYTHON" "$@"; '
                'else exec "$LZ_PYTHON" "$@"; fi')


def build_command(mode: str, nproc: int, rest: list[str], nnodes: int = 1, node_rank: int = 0,
                  master_addr: str = "127.0.0.1", master_port: int | None = None,
                  timeout_s: int = 3600, gdbserver_port: int | None = None) -> list[str]:
    port = master_port or _free_port()
    cmd = ["timeout", "-k", "60", str(timeout_s), sys.executable, "-m", "torch.distributed.run",
           f"--nnodes={nnodes if mode == 'node' else 1}", f"--nproc-per-node={nproc}",
           f"--master-addr={master_addr if mode == 'node' else '127.0.0.1'}", f"--master-port={port}"]
    if mode == "node":
        cmd.append(f"--node-rank={node_rank}")
    if gdbserver_port:
        # torchrun then runs `bash -c WRAPPER lz-rank <python args>` in every rank
        cmd += ["--no-python", "bash", "-c", _GDB_WRAPPER, "lz-rank"]
    return cmd + rest


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("mode", choices=["local", "node"])
    ap.add_argument("nproc", type=int)
    ap.add_argument("--nnodes", type=int, default=1)
    ap.add_argument("--node-rank", type=int, default=0)
    ap.add_argument("--master-addr", default="127.0.0.1")
    ap.add_argument("--master-port", type=int, default=None)
    ap.add_argument("--timeout", type=int, default=3600)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--gdbserver", type=int, default=None, metavar="PORT",
                    help="run rank 0 under gdbserver listening on PORT")
    a, rest = ap.parse_known_args(argv)
    cmd = build_command(a.mode, a.nproc, rest, a.nnodes, a.node_rank, a.master_addr, a.master_port, a.timeout,
                        gdbserver_port=a.gdbserver)
    env = dict(os.environ)
    env.setdefault("NCCL_DEBUG", "WARN")
    if a.gdbserver:
        env["LZ_GDB_PORT"] = str(a.gdbserver)
        env["LZ_PYTHON"] = sys.executable
    if a.dry_run:
        print(shlex.join(cmd))
        return 0
    if a.gdbserver and not shutil.which("gdbserver"):
        print("gdbserver is not installed on this machine", file=sys.stderr)
        return 2
    return subprocess.call(cmd, env=env)


if __name__ == "__main__":
    sys.exit(main())
