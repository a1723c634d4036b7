"""The benchmark's configurations are valid on CPU: every (config, N) builds its layouts
(on the meta device), the assignment covers every rollout worker's entries exactly, and the
devices and engines are consistent; the roofline arithmetic and the reference arm's line."""
import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

from weightbridge_b200 import WeightData  # noqa: E402
from weightbridge_b200.control.assign import assign_sources, restrict  # noqa: E402
from weightbridge_b200.core.shard import covered_numel, shard_numel  # noqa: E402
from weightbridge_b200.models.arch import get_arch  # noqa: E402
from weightbridge_b200.parallel.megatron import MegatronLayout  # noqa: E402
from weightbridge_b200.parallel.sglang import SGLangLayout  # noqa: E402

CASES = [("llama8b", 1), ("llama8b", 2), ("llama8b", 4), ("llama8b", 8), ("llama8b-fanout", 8),
         ("llama8b-broadcast", 4), ("llama8b-broadcast", 8),
         ("qwen3-moe-fp8", 8), ("qwen3-moe-fp8-etp", 8), ("llama70b-colocated", 8), ("deepseek-lite-fp8", 4),
         ("deepseek-lite-fp8", 8)]


def _meta(lay):
    return lay.to_wb(lay.allocate(device="meta", dtype=torch.bfloat16, fill=False))[0]


@pytest.mark.parametrize("config,n", CASES)
def test_bench_scenario_is_consistent(config, n):
    model, roles, desc = bench.scenario(config, n)
    arch = get_arch(model)
    assert all(0 <= r.device < n for r in roles) and {r.device for r in roles} == set(range(n))
    hosts = [r for r in roles if r.kind == "rollout" and r.host]
    assert {r.engine for r in hosts} == {r.engine for r in roles if r.kind == "rollout"}
    smetas = [_meta(MegatronLayout(arch, **r.layout)) for r in roles if r.kind == "trainer"]
    rmetas = {i: _meta(SGLangLayout(arch, **r.layout)) for i, r in enumerate(roles) if r.kind == "rollout"}
    plan = assign_sources(smetas, rmetas)
    for r, meta in rmetas.items():
        # every element of every (non-scale) entry's shards arrives from exactly one sender
        weights = [n for n in meta.names() if (meta.quant(n) or {}).get("role") != "scale"]
        got = 0
        for s, targets in plan.items():
            names = targets.get(r, [])
            if names:
                ov = WeightData.compute_overlap(restrict(smetas[s], names), meta)
                got += sum(covered_numel(reg, meta.shards(n)) for n, regs, _dt in ov if n in names for reg in regs)
        want = sum(shard_numel(sh) for n in weights for sh in meta.shards(n))
        assert got == want, (config, n, r, got, want)


def test_roofline_fractions():
    peak, source = bench._peer_peak()
    assert source.startswith("measured") and 700 < peak < 900     # profiles/nvlink_peer_peak.json
    # two TP pairs: each sender's link carries peak * 5 ms worth of bytes
    n = int(peak * 1e9 * 5e-3)
    routes = [{"src": 0, "dst": [2], "bytes": n, "multicast": False}, {"src": 1, "dst": [3], "bytes": n, "multicast": False}]
    rf = bench._roofline(routes, bytes_read=2 * n, payload=2 * n, ms=5.0)
    assert rf["bound"].startswith("nvlink") and rf["fraction_of_measured"] == 1.0
    hbm = bench._measured_peaks().get("hbm_gbs", 6650.0)
    local = [{"src": 0, "dst": [0], "bytes": int(hbm * 1e9 / 2), "multicast": False}]
    rf = bench._roofline(local, bytes_read=hbm * 1e9 / 2, payload=hbm * 1e9 / 2, ms=1000.0)
    assert rf["bound"].startswith("hbm") and rf["fraction_of_measured"] == 1.0


def test_link_bytes_unicast_fanout_and_multicast():
    """One sender to three replicas: unicast leaves the sender's GPU three times, multicast
    once; each replica's GPU takes the bytes in once either way; a route to the sender's own
    GPU stays in HBM."""
    uni = [{"src": 0, "dst": [d], "bytes": 10, "multicast": False} for d in (1, 2, 3)]
    eg, mc, ing, local = bench._link_bytes(uni + [{"src": 0, "dst": [0], "bytes": 7, "multicast": False}])
    assert eg == {0: 30} and mc == {} and ing == {1: 10, 2: 10, 3: 10} and local == 7
    mcr = [{"src": 0, "dst": [1, 2, 3], "bytes": 10, "multicast": True}]
    eg, mc, ing, local = bench._link_bytes(mcr)
    assert eg == {} and mc == {0: 10} and ing == {1: 10, 2: 10, 3: 10} and local == 0
    peak, _ = bench._peer_peak()
    n = int(peak * 1e6)                      # 1 ms of the peer peak
    rf = bench._roofline([dict(r, bytes=n) for r in uni], bytes_read=3 * n, payload=3 * n, ms=3.0)
    assert "egress of GPU 0" in rf["bound"] and rf["fraction_of_measured"] == 1.0
    # multicast egress is divided by the multicast store peak (at most the peer peak)
    mc_peak, _ = bench._mc_peak(peak)
    rf = bench._roofline([dict(mcr[0], bytes=n)], bytes_read=n, payload=3 * n, ms=1.0)
    assert rf["multicast_peak_gbs"] == mc_peak and abs(rf["ideal_ms"] - peak / mc_peak) < 1e-3


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and ("unavailable" in line or "value" in line)


def _join(init, idx, nprocs, q):
    import os
    os.environ["TORCHELASTIC_USE_AGENT_STORE"] = "True"       # what torchrun sets in every rank
    import torch.distributed as dist
    bench._init_group(init, idx, nprocs, timeout_s=30)
    dist.barrier()
    q.put(idx)
    dist.destroy_process_group()


def test_job_group_forms_with_more_processes_than_torchrun_ranks():
    """The bench's job-wide group (16 processes on 8 torchrun ranks for the colocated 70B
    layout) forms under torchrun's environment: process 0 serves the store itself."""
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_join, args=(f"tcp://127.0.0.1:{port}", i, 3, q)) for i in range(3)]
    for p in ps:
        p.start()
    got = sorted(q.get(timeout=60) for _ in ps)
    for p in ps:
        p.join(30)
    assert got == [0, 1, 2] and all(p.exitcode == 0 for p in ps)
