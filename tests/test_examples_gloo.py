"""The RL weight-sync example runs end to end on CPU (gloo) ranks through the
host transport: every version reaches every inference rank bit-exactly and
the periodic dump is readable."""
import pytest

from tests._mp import run_ranks


def _worker(rank, world, mode, dump_dir):
    from results_b200.examples import rl_weight_sync
    from results_b200.parallel import weights

    ok = rl_weight_sync.main(["--device", "cpu", "--small", "--layers", "2", "--steps", "3", "--mode", mode,
                              "--dump-dir", dump_dir, "--dump-every", "2"])
    import torch.distributed as dist

    dist.barrier()
    back = weights.load_dump(dump_dir, 2)
    return ok, len(back)


@pytest.mark.parametrize("mode", ["raw", "split_ans"])
def test_rl_weight_sync_example_cpu(mode, tmp_path):
    res = run_ranks(_worker, 3, args=(mode, str(tmp_path)))
    assert all(ok and n > 0 for ok, n in res), res


def _resume_worker(rank, world, dump_dir):
    import torch

    from results_b200.examples import rl_weight_sync
    from results_b200.parallel import weights

    common = ["--device", "cpu", "--small", "--layers", "2", "--mode", "split_ans", "--dump-dir", dump_dir,
              "--dump-every", "1"]
    ok1 = rl_weight_sync.main(common + ["--steps", "2"])
    import torch.distributed as dist

    dist.barrier()
    ok2 = rl_weight_sync.main(common + ["--steps", "1", "--resume"])  # continues as version 3
    dist.barrier()
    v = weights.latest_dump_version(dump_dir)
    # version 3 was produced from version 2 by step 3's update: it differs from 2
    a, b = weights.load_dump(dump_dir, 2), weights.load_dump(dump_dir, 3)
    changed = any(not torch.equal(a[k].view(torch.uint8), b[k].view(torch.uint8)) for k in a)
    return ok1, ok2, v, changed


def test_rl_weight_sync_resume(tmp_path):
    res = run_ranks(_resume_worker, 2, args=(str(tmp_path),))
    assert all(r == (True, True, 3, True) for r in res), res
