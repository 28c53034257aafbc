"""Public weight-update API on CPU tensors (gloo ranks): send_weights /
recv_weights / broadcast_weights through the host transport, raw and
LZC1-encoded, receivers bit-identical to the sender and to its dump."""
import pytest

from tests._mp import run_ranks


def _state_dict(seed, empty=False):
    import torch

    g = torch.Generator().manual_seed(seed)
    sd = {
        "embed.weight": (torch.randn(3001, 64, generator=g) * 0.02).to(torch.bfloat16),
        "layers.0.norm.weight": torch.ones(64, dtype=torch.bfloat16),
        "layers.0.mlp.weight": (torch.randn(64, 257, generator=g) * 0.02).to(torch.float32),
        "layers.0.fp8.weight": (torch.randn(4096, generator=g) * 0.5).to(torch.float8_e4m3fn),
    }
    if empty:
        sd = {k: torch.zeros_like(v) for k, v in sd.items()}
    return sd


def _worker(rank, world, mode, dump_dir):
    import torch

    from results_b200.parallel import weights

    ref = _state_dict(11)
    out = []
    # point to point, in small buckets (several per call)
    sd = ref if rank == 0 else _state_dict(0, empty=True)
    if rank == 0:
        weights.send_weights(sd, list(range(1, world)), mode=mode, bucket_bytes=64 << 10, dump_dir=dump_dir,
                             weight_version=5)
    else:
        weights.recv_weights(sd, 0, mode=mode, bucket_bytes=64 << 10)
    same = lambda a, b: torch.equal(a.view(torch.uint8), b.view(torch.uint8))  # noqa: E731
    out.append(all(same(sd[k], ref[k]) for k in ref))
    # broadcast from the last rank
    src = world - 1
    sd2 = ref if rank == src else _state_dict(0, empty=True)
    weights.broadcast_weights(sd2, src=src, mode=mode)
    out.append(all(same(sd2[k], ref[k]) for k in ref))
    import torch.distributed as dist

    dist.barrier()
    back = weights.load_dump(dump_dir, 5)
    out.append(all(same(back[k], ref[k]) for k in ref))
    return out


@pytest.mark.parametrize("mode", ["raw", "split_ans"])
def test_weights_api_on_cpu_tensors(mode, tmp_path):
    res = run_ranks(_worker, 3, args=(mode, str(tmp_path)))
    assert all(all(r) for r in res), res
