"""RL weight-update transfer across real GPUs: point-to-point and NVLS
broadcast, raw and split+rANS, partial encode fractions; receivers must end
bit-identical to the sender (checked against the safetensors dump oracle)."""
import pytest
import torch

from tests._mp import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _small_specs():
    from results_b200.models.shapes import glm4_9b_specs

    return glm4_9b_specs(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1000, vocab=5003)


def _worker(rank, world, cases, dump_dir):
    import torch

    from results_b200.config import Config
    from results_b200.models.shapes import make_state_dict
    from results_b200.parallel.comm import Communicator
    from results_b200.parallel import weights

    comm = Communicator(config=Config(user_bytes=96 << 20, stage_bytes=512 << 20, timeout_s=20.0))
    specs = _small_specs()
    ref = make_state_dict(specs, seed=7)
    results = []
    for mode, kind, frac in cases:
        wt = weights.WeightTransfer(comm, mode=mode, encode_fraction=frac, nblocks=64, kslots=3)
        if rank == 0:
            sd = ref
        else:
            sd = make_state_dict(specs, empty=True)
            for t in sd.values():
                t.fill_(-7)
        if kind == "p2p":
            if rank == 0:
                for d in range(1, world):
                    wt.send(list(sd.values()), d)
            else:
                wt.recv(list(sd.values()), 0)
        else:
            wt.broadcast(list(sd.values()), 0)
        torch.cuda.synchronize()
        comm.check()
        ok = all(torch.equal(sd[k].view(torch.int16), ref[k].view(torch.int16)) for k in ref)
        results.append((mode, kind, frac, ok))
    # zero-copy raw broadcast into symmetric destinations
    comm.reset_alloc()
    sym = [comm.empty(t.shape, t.dtype) for t in ref.values()]
    for t in sym:
        t.fill_(-3)
    wt = weights.WeightTransfer(comm, mode="raw")
    for kernel_path in (False, True):  # the default (copy engines / relay), then the sender-store kernel
        kw = {"relay": False, "copy_engine": False} if kernel_path else {}
        wt.broadcast_direct(sym, 0, src_tensors=list(ref.values()) if rank == 0 else None, nblocks=32, **kw)
    torch.cuda.synchronize()
    comm.check()
    bad_idx = [i for i, (a, b) in enumerate(zip(sym, ref.values()))
               if not torch.equal(a.view(torch.int16), b.view(torch.int16))]
    diag = ""
    if bad_idx:
        a, b = sym[bad_idx[0]].view(-1).view(torch.int16), list(ref.values())[bad_idx[0]].view(-1).view(torch.int16)
        first = int((a != b).nonzero()[0].item())
        diag = (f"rank {rank}: {len(bad_idx)}/{len(sym)} tensors differ; first tensor {bad_idx[0]} "
                f"numel {a.numel()} first diff at {first} got {int(a[first])} want {int(b[first])} "
                f"ptr%16={sym[bad_idx[0]].data_ptr() % 16}")
    results.append(("raw", "direct", diag, not bad_idx))
    # public API: broadcast_weights of a symmetric state_dict takes the zero-copy path
    sym_sd = {k: comm.empty(t.shape, t.dtype) for k, t in ref.items()}
    for k, t in sym_sd.items():
        if rank == 0:
            t.copy_(ref[k])
        else:
            t.fill_(-5)
    weights.broadcast_weights(sym_sd, 0, comm=comm, mode="raw")
    torch.cuda.synchronize()
    comm.check()
    results.append(("raw", "broadcast_weights_symmetric", 0.0,
                    all(torch.equal(sym_sd[k].view(torch.int16), ref[k].view(torch.int16)) for k in ref)))
    # copy-engine DMA 0 -> 1 into symmetric tensors (twice: the pair sequence moves on)
    ce = [comm.empty(t.shape, t.dtype) for t in ref.values()]
    for t in ce:
        t.fill_(-2)
    for _ in range(2):
        wt.send_copy_engine(ce, 0, 1, src_tensors=list(ref.values()) if rank == 0 else None)
    torch.cuda.synchronize()
    comm.check()
    if rank == 1:
        results.append(("raw", "copy_engine", 0.0,
                        all(torch.equal(a.view(torch.int16), b.view(torch.int16)) for a, b in zip(ce, ref.values()))))
    # staged broadcast into ordinary (non-symmetric) tensors, twice in a row, with
    # a stage smaller than the largest tensor (pieces, several buckets, both buffers)
    plain = make_state_dict(specs, empty=True) if rank != 0 else None
    if rank != 0:
        for t in plain.values():
            t.fill_(-9)
    for _ in range(2):
        wt.broadcast_staged(list((ref if rank == 0 else plain).values()), 0, stage_bytes=1 << 20)
    torch.cuda.synchronize()
    comm.check()
    if rank != 0:
        results.append(("raw", "staged", 0.0,
                        all(torch.equal(plain[k].view(torch.int16), ref[k].view(torch.int16)) for k in ref)))
    # dump oracle: rank 0 dumps, the others compare what they received with it
    if rank == 0:
        weights.dump_tensors(list(ref.items()), dump_dir, 3, 0, group_name="test")
    import torch.distributed as dist

    dist.barrier()
    if rank != 0:
        back = weights.load_dump(dump_dir, 3)
        results.append(("dump", "oracle", 1.0,
                        all(torch.equal(back[k].cuda().view(torch.int16), ref[k].view(torch.int16)) for k in ref)))
    comm.close()
    return results


CASES = [("raw", "p2p", 0.0), ("split_ans", "p2p", 1.0), ("split_ans", "bcast", 1.0),
         ("raw", "bcast", 0.0), ("split_ans", "bcast", 0.4), ("split_ans", "p2p", 0.6)]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_weight_transfer(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = run_ranks(_worker, world, backend="nccl", args=(CASES, str(tmp_path)), timeout=600)
    bad = [r for rr in res for r in rr if not r[3]]
    assert not bad, bad
