"""Host-side tools: log parsers, launcher command, SVG plots, CSV schemas, config."""
import csv
import os

from results_b200.utils import csvfmt, logparse, plots


def test_logparse_reference_and_own_lines():
    lines = [
        "[E] DietGPUCompressorBackend: Compressed 1048576 bytes to 700000 bytes, ratio 0.6676 weight=q_proj",
        "[E] DietGPUCompressorBackend: Compressed 1048576 bytes to 702000 bytes, ratio 0.6695 weight=q_proj",
        logparse.log_line("mlp.down_proj.weight", 2000, 1350),
        "unrelated line",
    ]
    s = logparse.by_size(lines)
    assert abs(s[1048576] - (700000 + 702000) / 2 / 1048576) < 1e-9
    w = logparse.by_weight(lines)
    assert "q_proj" in w and "mlp.down_proj.weight" in w


def test_launch_command():
    from results_b200.launch import build_command

    cmd = build_command("local", 8, ["bench.py", "--gpus", "8"], master_port=29555)
    assert "--nproc-per-node=8" in cmd and "--master-addr=127.0.0.1" in cmd and cmd[:2] == ["timeout", "-k"]
    cmd2 = build_command("node", 8, ["x.py"], nnodes=2, node_rank=1, master_addr="10.0.0.2", master_port=1)
    assert "--nnodes=2" in cmd2 and "--node-rank=1" in cmd2


def test_schema_a_csv_and_chart(tmp_path):
    rows = []
    for v, base in (("P2P", 1.0), ("NVLS", 1.2)):
        for s in (1 << 20, 1 << 24, 1 << 30):
            for m in ("wall_ms", "cuda_ms"):
                rows.append({"metric": m, "size_label": csvfmt.size_label(s), "size_bytes": s, "world_size": 8,
                             "variant": v, "nccl_ms": 1.0, "variant_ms": base, "variant_vs_nccl_pct": 100,
                             "nccl_algbw_GBps": 1, "variant_algbw_GBps": s / base / 1e6,
                             "nccl_busbw_GBps": 1, "variant_busbw_GBps": s / base / 1e6 * 1.75, "comp_ratio": ""})
    p = str(tmp_path / "a.csv")
    csvfmt.write_rows(p, csvfmt.SCHEMA_A, rows, blocks=[[r for r in rows if r["metric"] == "wall_ms"],
                                                       [r for r in rows if r["metric"] == "cuda_ms"]])
    with open(p) as f:
        assert f.readline().strip().split(",") == csvfmt.SCHEMA_A
    svg = plots.sweep_chart(p, str(tmp_path / "a.svg"))
    assert open(svg).read().startswith("<svg")


def test_config_env(monkeypatch):
    from results_b200.config import Config

    monkeypatch.setenv("LZ_TIMEOUT_S", "3.5")
    monkeypatch.setenv("RING_NUM_CHANNELS", "2")
    monkeypatch.setenv("HD_MAX_MB", "64")
    c = Config.from_env()
    assert c.timeout_s == 3.5 and c.ring_channels == 2 and c.hd_max_bytes == 64 << 20


def test_size_labels():
    assert csvfmt.size_label(1 << 30) == "1 GB" and csvfmt.size_label(1024) == "1 KB"


def test_trace_ranges_and_bucket_logs(caplog):
    """Tracing is a no-op unless enabled; enabled ranges nest without a GPU
    profiler attached; bucket log lines carry tensor and byte counts."""
    import logging

    import torch

    from results_b200.parallel import weights
    from results_b200.utils import trace

    calls = []

    @trace.traced("probe")
    def f(x, algo=None):
        calls.append(x)
        return x + 1

    assert f(1) == 2
    trace.enable(True)
    try:
        if torch.cuda.is_available():
            assert f(2, algo="ll") == 3
    finally:
        trace.enable(False)
    with caplog.at_level(logging.INFO, logger="results_b200"):
        weights._log_bucket("send", 3, [("a", torch.zeros(1024)), ("b", torch.zeros(256, dtype=torch.bfloat16))])
    assert any("[BUCKET] send 3 start tensors=2" in r.getMessage() for r in caplog.records)


def test_size_table_choices():
    """The measured size table: ll for small messages, one-shot, then two-shot,
    NVLS or the copy-engine two-shot by world; the copy-engine path only for
    symmetric out-of-place buffers; exact mode never picks NVLS; unaligned
    sizes never get a vector-only algorithm."""
    from results_b200.parallel.tuning import choose

    KB, MB = 1 << 10, 1 << 20
    assert choose(1 * KB, 2, True, True) == "ll"
    assert choose(256 * KB, 2, True, True) == "ll"
    assert choose(4 * MB, 2, True, True) == "oneshot"
    assert choose(64 * MB, 2, True, True) == "twoshot"
    assert choose(1 << 30, 2, True, True) == "ce"
    assert choose(1 << 30, 2, True, True, out_of_place=False) == "twoshot"
    assert choose(1 << 30, 2, True, False) == "twoshot"
    assert choose(512 * MB, 4, True, True) == "nvls"
    assert choose(512 * MB, 4, True, True, exact=True) == "ce"
    assert choose(64 * MB, 8, True, True, exact=True) == "twoshot"
    assert choose(1 << 30, 4, True, True) == "ce"
    assert choose(128 * KB, 8, True, True) == "ll"
    assert choose(512 * KB, 8, True, True) == "oneshot"
    assert choose(4 * MB, 8, True, True) == "twoshot"
    assert choose(64 * MB, 8, True, True) == "nvls"
    assert choose(64 * MB, 8, False, True) == "twoshot"
    assert choose(64 * MB, 4, True, True) == "twoshot"
    assert choose(1000 * 2 + 2, 8, True, True) == "oneshot"  # not a multiple of 16 bytes


def test_bench_baseline_ratio_uses_aggregates():
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(root, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert abs(m.REF_AGGREGATE_1GB[8] - 53.60 * 8) < 1e-9
    assert abs(m.REF_AGGREGATE_1GB[2] - 54.68 * 2) < 1e-9
    assert 1 not in m.REF_AGGREGATE_1GB and 4 not in m.REF_AGGREGATE_1GB


def test_config_env_and_bounds_library_name(monkeypatch):
    from results_b200.config import Config
    from results_b200.utils import build

    monkeypatch.setenv("LZ_RATIO_BUDGET", "0.7")
    assert Config.from_env().ratio_budget == 0.7
    monkeypatch.setenv("LZ_BOUNDS", "1")
    assert build.cuda_lib_name() == "liblz_cuda_bounds.so"
    monkeypatch.setenv("LZ_BOUNDS", "0")
    assert build.cuda_lib_name() == "liblz_cuda.so"
    # the heap holds flags, one-shot buffers, low-latency areas, stage and user region
    c = Config(user_bytes=64 << 20, stage_bytes=32 << 20, oneshot_bytes=4 << 20)
    assert c.total_heap_bytes() >= (1 << 20) + 2 * (4 << 20) + (8 << 20) + (32 << 20) + (64 << 20)


def test_launch_gdbserver_wraps_rank0_only(tmp_path):
    """--gdbserver runs rank 0 under gdbserver and the others plainly: the
    wrapper is checked by running it with a fake gdbserver on PATH."""
    import os
    import subprocess
    import sys

    from results_b200 import launch

    cmd = launch.build_command("local", 2, ["-c", "print(1)"], gdbserver_port=1234)
    i = cmd.index("--no-python")
    assert cmd[i + 1:i + 5] == ["bash", "-c", launch._GDB_WRAPPER, "lz-rank"]
    fake = tmp_path / "gdbserver"
    fake.write_text("#!/bin/sh\necho gdbserver \"$@\"\n")
    fake.chmod(0o755)
    base = dict(os.environ, PATH=f"{tmp_path}:{os.environ['PATH']}", LZ_GDB_PORT="1234", LZ_PYTHON=sys.executable)
    out0 = subprocess.run(["bash", "-c", launch._GDB_WRAPPER, "lz-rank", "-c", "print('rank')"],
                          env=dict(base, RANK="0"), capture_output=True, text=True).stdout
    out1 = subprocess.run(["bash", "-c", launch._GDB_WRAPPER, "lz-rank", "-c", "print('rank')"],
                          env=dict(base, RANK="1"), capture_output=True, text=True).stdout
    assert out0.startswith("gdbserver :1234 ") and out1.strip() == "rank"


def test_result_charts(tmp_path):
    """Grouped bars, KV latency and log-scale latency charts render valid SVG."""
    import json

    from results_b200.utils import csvfmt, plots

    kv = tmp_path / "kv.csv"
    kv.write_text("Input Token,nccl kv cache transfer latency (ms),ours_ce latency (ms)\n"
                  "7680,2.7,0.8\n102400,8.3,6.0\n")
    assert plots.kv_chart(str(kv), str(tmp_path / "kv.svg")).endswith("kv.svg")
    wj = tmp_path / "w.json"
    wj.write_text(json.dumps({"model": "glm4-9b", "world": 2, "results": {"a": {"sec": 0.03}, "b": {"sec": 0.02}}}))
    svg = open(plots.weight_update_chart([str(wj)], str(tmp_path / "w.svg"))).read()
    assert svg.startswith("<svg") and svg.count("<rect") >= 3
    rows = [{"metric": "cuda_ms", "size_label": "1 KB", "size_bytes": 1024, "world_size": 2, "variant": v,
             "variant_ms": ms} for v, ms in (("NCCL", 0.0145), ("LL", 0.0043))]
    rows += [{**r, "size_bytes": 2048, "size_label": "2 KB"} for r in rows]
    sweep = tmp_path / "a.csv"
    csvfmt.write_rows(str(sweep), csvfmt.SCHEMA_A, rows)
    assert "us (log)" in open(plots.sweep_latency_chart(str(sweep), str(tmp_path / "l.svg"))).read()


def test_low_latency_flag_values():
    """The low-latency one-shot's call flags (odd-multiplier hash of the call
    number, low bit set; the same formula as ll_flag in csrc/lz_allreduce.cu)
    are never 0 (zeroed memory) and never repeat within 2^31 uses of one
    parity area, so a stale word can never carry the current flag."""
    import numpy as np

    e = np.arange(0, 1 << 22, dtype=np.uint64)
    f = (((e + 1) * np.uint64(0x9E3779B1)) & np.uint64(0xFFFFFFFF)) | np.uint64(1)
    assert (f != 0).all()
    for parity in (0, 1):
        v = f[parity::2]
        assert np.unique(v).size == v.size
    import re

    src = open(__import__("os").path.join(__import__("os").path.dirname(__file__), "..", "csrc",
                                          "lz_allreduce.cu")).read()
    assert re.search(r"\(uint32_t\)\(epoch \+ 1ull\) \* 0x9E3779B1u\) \| 1u", src)


def test_clock_sampler_with_fake_nvml(monkeypatch):
    """Clock sampling reads NVML only (a fake module here): median SM clock of
    the busy samples, the union of event reasons, idle samples ignored."""
    import sys
    import time
    import types

    from results_b200.utils import clocks

    state = {"i": 0}
    seq = [(1965, 0x0), (1800, 0x4), (1900, 0x4), (300, 0x1)]  # busy, power cap, power cap, idle

    def clock(h, which):
        return seq[state["i"] % len(seq)][0]

    def reasons(h):
        r = seq[state["i"] % len(seq)][1]
        state["i"] += 1
        return r

    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0, nvmlInit=lambda: None, nvmlDeviceGetHandleByIndex=lambda d: d,
        nvmlDeviceGetMaxClockInfo=lambda h, w: 1965, nvmlDeviceGetClockInfo=clock,
        nvmlDeviceGetPowerUsage=lambda h: 700_000, nvmlDeviceGetCurrentClocksEventReasons=reasons)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    s = clocks.ClockSampler([0], period_s=0.001).start()
    while state["i"] < 8:
        time.sleep(0.001)
    summ = s.stop().summary()
    assert summ["sm_max_mhz"] == 1965 and summ["samples"] >= 8
    assert summ["reasons"] == ["sw_power_cap"]
    assert 1800 <= summ["sm_mhz"] <= 1965
    assert clocks.decode_reasons(0x8 | 0x40) == ["hw_slowdown", "hw_thermal_slowdown"]


def test_report_regenerates_quoted_tables():
    """The summary tables are regenerated from the committed measurements, and
    the headline claim (auto >= NCCL at every size and rank count) holds in
    the data."""
    import os

    from results_b200.utils import report

    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "results")
    text = report.main([root])
    assert "| 1 GB |" in text and "Weight update" in text
    import glob
    import re

    for p in glob.glob(os.path.join(root, "csv", "allreduce_sweep_*xB200_graph.csv")):
        d = report.sweep_times(p)
        for size, r in d.items():
            assert r["Auto"] <= r["NCCL"] * 1.0001, (p, size, r["Auto"], r["NCCL"])
    assert re.search(r"Smallest margin over NCCL: 1\.\d\dx", text)


def test_public_api_names_resolve():
    """Every name the package advertises resolves (lazily) on a CPU-only box."""
    import results_b200 as lz

    for name in lz.__all__:
        assert getattr(lz, name) is not None, name
    assert "allreduce" in dir(lz)
