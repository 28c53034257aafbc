"""The range-checked debug build (LZ_BOUNDS=1, liblz_cuda_bounds.so) runs the
emulated multi-rank kernels without a false bounds report and bit-identical
to the release build's results."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import torch
from results_b200 import _native
from results_b200.parallel.emulate import EmulatedWorld
assert _native.cuda()._name.endswith("liblz_cuda_bounds.so"), _native.cuda()._name
R = 4
w = EmulatedWorld(R, heap_bytes=96 << 20, stage_bytes=32 << 20)
g = torch.Generator(device="cuda").manual_seed(3)
n = 40000
xs = [(torch.randn(n, device="cuda", generator=g) * 1e-2).to(torch.bfloat16) for _ in range(R)]
ref = xs[0].float().clone()
for x in xs[1:]:
    ref += x.float()
ref = ref.to(torch.bfloat16)
for algo in ("ll", "oneshot", "twoshot"):
    outs = [torch.empty_like(x) for x in xs]
    w.allreduce(xs, outs, algo, nblocks=4, nthreads=256)
    torch.cuda.synchronize()
    for r in range(R):
        assert w.status(r) == 0, (algo, r, hex(w.status(r)))
        assert torch.equal(outs[r], ref), (algo, r)
m = 8 * 4096 * R
ins = [torch.randn(m, device="cuda", generator=g).to(torch.bfloat16) for _ in range(R)]
outs = [torch.zeros_like(x) for x in ins]
w.all_to_all(ins, outs, compress=True, nblocks=4)
torch.cuda.synchronize()
for r in range(R):
    assert w.status(r) == 0
    want = torch.cat([ins[s].view(R, -1)[r] for s in range(R)])
    assert torch.equal(outs[r], want)
w.close()
print("bounds ok")
"""


def test_bounds_checked_build_runs_clean():
    env = dict(os.environ, LZ_BOUNDS="1")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
    proc = subprocess.run([sys.executable, "-c", SCRIPT], env=env, cwd=root, capture_output=True, text=True,
                          timeout=600)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    assert "bounds ok" in proc.stdout
