"""Green-context SM budgets: kernels launched on the budget's stream run on
at most the granted SMs; topology probes report the B200."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sms", [16, 32])
def test_green_context_limits_sms(sms):
    from results_b200.utils.sm_budget import SmBudget, probe_smids

    with SmBudget(0, sms) as b:
        assert b.sm_count >= sms
        ids = probe_smids(b.stream, nblocks=512)
        assert min(ids) >= 0
        assert len(set(ids)) <= b.sm_count
    # a full-device launch spreads further
    ids_all = probe_smids(torch.cuda.current_stream(), nblocks=512)
    assert len(set(ids_all)) > sms


def test_codec_runs_inside_budget():
    from results_b200.ops import codec
    from results_b200.utils.sm_budget import SmBudget

    x = (torch.randn(1 << 20, device="cuda") * 0.02).to(torch.bfloat16)
    with SmBudget(0, 32) as b:
        with torch.cuda.stream(b.stream):
            blob = codec.encode(x, nblocks=32 * 3)
            y = codec.decode(blob, like=x)
        b.stream.synchronize()
    assert torch.equal(x.view(torch.int16), y.view(torch.int16))


def test_topology_probe():
    from results_b200.utils import topology

    info = topology.device_info(0)
    assert info["sm_count"] >= 100 and info["cc"].startswith("10.")
    s = topology.summary()
    assert len(s["devices"]) == torch.cuda.device_count()
