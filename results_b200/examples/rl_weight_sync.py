"""RL weight synchronisation loop: a trainer rank updates its weights every
step and pushes them to the inference ranks, which check what they received.

    torchrun --nproc-per-node 8 -m results_b200.examples.rl_weight_sync --steps 5
    torchrun --nproc-per-node 3 -m results_b200.examples.rl_weight_sync --device cpu --layers 2

With ``--resume`` the trainer restarts from the newest dumped version
(checkpoint / resume of the weight stream).

Rank 0 plays the trainer (GLM-4-9B-shaped state_dict, optionally fewer
layers), every other rank an inference engine holding its own copy. Each step
the trainer applies a synthetic optimizer update, then every rank calls
``broadcast_weights`` (CUDA: native kernels; with ``--symmetric`` the weights
live in the symmetric heap and the update is zero-copy; CPU: the host
transport). Receivers compare a checksum of what they hold with the
trainer's; every ``--dump-every`` versions the trainer also dumps the
weights (safetensors + manifest) as the reference's updater does
(back_up/update_weight_from_distributed.py:92-160, 345-357).
"""
from __future__ import annotations

import argparse
import datetime
import os
import time

import torch
import torch.distributed as dist


def checksum(sd) -> int:
    s = 0
    for t in sd.values():
        v = t.reshape(-1).view(torch.uint8).to(torch.int64)
        s = (s * 1000003 + int((v * torch.arange(1, v.numel() + 1, dtype=torch.int64, device=v.device)).sum())) \
            % (1 << 61)
    return s


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--mode", default="raw", choices=["raw", "split_ans"])
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"])
    ap.add_argument("--symmetric", action="store_true", help="weights in the symmetric heap (zero-copy update)")
    ap.add_argument("--dump-dir", default=None)
    ap.add_argument("--dump-every", type=int, default=0)
    ap.add_argument("--small", action="store_true", help="tiny shapes (tests)")
    ap.add_argument("--resume", action="store_true",
                    help="trainer starts from the newest version dumped in --dump-dir")
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    cuda = a.device == "cuda"
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    if not dist.is_initialized():
        dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=300),
                                **({"device_id": torch.device("cuda", torch.cuda.current_device())} if cuda else {}))
    from results_b200.models.shapes import glm4_9b_specs, make_state_dict
    from results_b200.parallel import weights

    specs = (glm4_9b_specs(layers=a.layers, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=1000)
             if a.small else glm4_9b_specs(layers=a.layers))
    dev = "cuda" if cuda else "cpu"
    sd = make_state_dict(specs, seed=1, empty=(rank != 0), device=dev)
    comm = None
    if cuda:
        import results_b200 as lz
        from results_b200.config import Config

        nbytes = sum(t.numel() * t.element_size() for t in sd.values())
        comm = lz.init(config=Config(user_bytes=nbytes + (64 << 20) if a.symmetric else 64 << 20))
        if a.symmetric:
            sym = {k: comm.empty(t.shape, t.dtype) for k, t in sd.items()}
            for k, t in sym.items():
                t.copy_(sd[k])
            sd = sym
    start = 1
    if a.resume and a.dump_dir:
        # every rank learns the version; the trainer loads its weights
        v = [weights.latest_dump_version(a.dump_dir) if rank == 0 else None]
        dist.broadcast_object_list(v, src=0)
        if v[0] is not None:
            if rank == 0:
                back = weights.load_dump(a.dump_dir, v[0])
                for k, t in sd.items():
                    t.copy_(back[k].to(t.device))
            start = v[0] + 1
    ok_all = True
    for step in range(start, start + a.steps):
        if rank == 0:  # a synthetic optimizer step: every weight moves a little
            g = torch.Generator(device=dev).manual_seed(step)
            for t in sd.values():
                if t.is_floating_point():
                    t.add_((torch.randn(t.shape, generator=g, device=dev) * 1e-3).to(t.dtype))
            if a.dump_dir and a.dump_every and step % a.dump_every == 0:
                weights.dump_tensors(list(sd.items()), a.dump_dir, step, 0, group_name="trainer")
                weights.mark_dump_complete(a.dump_dir, step, 1)
        want = [checksum(sd) if rank == 0 else None]
        t0 = time.perf_counter()
        weights.broadcast_weights(sd, src=0, comm=comm, mode=a.mode)
        if cuda:
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        dist.broadcast_object_list(want, src=0)
        ok = checksum(sd) == want[0]
        flag = torch.tensor([0 if ok else 1], device=dev)  # NCCL reduces device tensors
        dist.all_reduce(flag)
        ok_all = ok_all and int(flag.item()) == 0
        if rank == 0:
            print(f"step {step}: weights v{step} on {world} ranks in {dt * 1e3:.1f} ms, "
                  f"all receivers bit-exact: {int(flag.item()) == 0}", flush=True)
    if comm is not None:
        import results_b200 as lz

        lz.shutdown()
    return ok_all


if __name__ == "__main__":
    ok = main()
    dist.destroy_process_group()
    raise SystemExit(0 if ok else 1)
