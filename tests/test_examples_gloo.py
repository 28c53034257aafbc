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
