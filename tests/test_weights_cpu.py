"""Host-side pieces of the weight-transfer engine (no GPU): encode-fraction
selection, bucketing by byte budget, model shapes and the dump manifest."""
import json
import os

import torch

from results_b200.models import shapes
from results_b200.parallel import weights


def test_encode_fraction_selection():
    for n in (1, 7, 10, 523):
        for f in (0.0, 0.2, 0.4, 0.6, 0.8, 1.0):
            flags = weights._encode_flags(n, f)
            assert sum(flags) == int(n * f)


def test_buckets_respect_budget():
    named = [(f"t{i}", torch.empty(1000 * (i % 5 + 1), dtype=torch.bfloat16)) for i in range(40)]
    out = list(weights.buckets(named, 6000))
    assert sum(len(b) for b in out) == 40
    for b in out:
        size = sum(t.numel() * 2 for _, t in b)
        assert size <= 6000 or len(b) == 1


def test_glm4_shapes_match_reference_rows():
    specs = {s.name: s for s in shapes.glm4_9b_specs()}
    # per-tensor sizes of csv/weight_update_rl_GLM4_9B.csv: gate_up 214 MB, down 107 MB, o/q 32 MB
    assert specs["model.layers.0.mlp.gate_up_proj.weight"].numel * 2 == 224_395_264
    assert specs["model.layers.0.mlp.down_proj.weight"].numel * 2 == 112_197_632
    assert specs["model.layers.0.self_attn.o_proj.weight"].numel * 2 == 33_554_432
    assert abs(shapes.total_params(list(specs.values())) / 1e9 - 9.4) < 0.05


def test_qwen_moe_shapes():
    specs = shapes.qwen35_a3b_specs()
    total = shapes.total_params(specs) / 1e9
    assert 30 < total < 40
    experts = [s for s in specs if "experts." in s.name]
    assert all(s.numel * 2 >= 64 << 20 for s in experts)  # coalesced >= 64 MB chunks


def test_dump_manifest_roundtrip(tmp_path):
    named = [("a.weight", torch.randn(8, 4).to(torch.bfloat16)), ("b.bias", torch.randn(3))]
    p = weights.dump_tensors(named, str(tmp_path), 12, 0, group_name="g")
    assert os.path.exists(p)
    rec = json.loads(open(os.path.join(tmp_path, "weight_version_000012", "manifest.jsonl")).readline())
    assert rec["num_tensors"] == 2 and rec["tensors"][0]["shape"] == [8, 4]
    back = weights.load_dump(str(tmp_path), 12)
    assert torch.equal(back["a.weight"].view(torch.int16), named[0][1].view(torch.int16))


def test_resume_skips_versions_whose_dump_did_not_complete(tmp_path):
    """A multi-shard dump cut short (no completion marker, or fewer shards
    than it promised) is never the version a resume picks."""
    d = str(tmp_path)
    t = [("w", torch.randn(4))]
    weights.dump_tensors(t, d, 1, 0)
    weights.dump_tensors(t, d, 1, 1)
    weights.mark_dump_complete(d, 1, 2)
    assert weights.latest_dump_version(d) == 1
    weights.dump_tensors(t, d, 2, 0)  # crash before shard 1 and the marker
    assert weights.latest_dump_version(d) == 1
    weights.mark_dump_complete(d, 2, 2)  # marker promising a shard the manifest lacks
    assert weights.latest_dump_version(d) == 1
    weights.dump_tensors(t, d, 2, 1)
    assert weights.latest_dump_version(d) == 2


def test_engine_cache_is_per_communicator_object():
    """Engines are cached per communicator object (not per id(), which a new
    communicator can reuse) and released with it."""
    import gc

    from results_b200.parallel import weights

    class FakeComm:
        rank, world, device, sm_count = 0, 1, 0, 148

    made = []
    orig = weights.WeightTransfer
    weights.WeightTransfer = lambda comm, mode, **kw: made.append(mode) or object()
    try:
        a = FakeComm()
        e1 = weights._engine(a, "raw")
        assert weights._engine(a, "raw") is e1
        assert weights._engine(a, "split_ans") is not e1
        del a
        gc.collect()
        b = FakeComm()
        weights._engine(b, "raw")
        assert len(made) == 3 and len(weights._ENGINES) == 1
    finally:
        weights.WeightTransfer = orig


def _fake_comm(world, rank=0, symmetric=True):
    import torch

    from results_b200.parallel import weights

    calls = []

    class Lib:
        def __getattr__(self, name):
            def f(*args):
                calls.append(name)
                return 0
            return f

    class Comm:
        pass

    c = Comm()
    c.world, c.rank, c.device, c.sm_count = world, rank, 0, 148
    c._lib = Lib()
    c.handle = None
    c._local_base = 0
    c.has_multicast = True
    c.is_symmetric = lambda t: symmetric
    wt = weights.WeightTransfer.__new__(weights.WeightTransfer)
    wt.comm, wt.pair_seq, wt.bcast_seq = c, {}, {}
    return wt, calls, torch


def test_zero_copy_dispatch_policy(monkeypatch):
    """broadcast_direct picks copy engines for 2 ranks with large tensors, the
    peer-store kernel for 2 ranks with small ones, and the relay for more."""
    import torch

    from results_b200.parallel import weights

    seen = []
    monkeypatch.setattr(weights.WeightTransfer, "send_copy_engine",
                        lambda self, d, src, dst, src_tensors=None: seen.append(("ce", src, dst)))
    monkeypatch.setattr(weights.WeightTransfer, "_direct_descs",
                        lambda self, d, s: (torch.zeros(1, dtype=torch.int64), len(d)))
    monkeypatch.setattr(weights, "_native", type("N", (), {"check": staticmethod(lambda rc, what: None)}))
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: type("S", (), {"cuda_stream": 0})())

    big = [torch.empty(0)] * 2
    monkeypatch.setattr(torch.Tensor, "numel", lambda self: 32 << 20, raising=False)
    wt, calls, _ = _fake_comm(2, rank=1)
    wt.broadcast_direct(big, 0)
    assert seen == [("ce", 0, 1)] and not calls

    monkeypatch.setattr(torch.Tensor, "numel", lambda self: 1 << 10, raising=False)
    seen.clear()
    wt, calls, _ = _fake_comm(2, rank=1)
    wt.broadcast_direct(big, 0)
    assert not seen and calls == ["lz_weight_transfer_direct"]

    wt, calls, _ = _fake_comm(8, rank=3)
    wt.broadcast_direct(big, 0)
    assert calls == ["lz_weight_broadcast_relay"]

    wt, calls, _ = _fake_comm(8, rank=3)
    wt.broadcast_direct(big, 0, relay=False, copy_engine=False)
    assert calls == ["lz_weight_transfer_direct"]
