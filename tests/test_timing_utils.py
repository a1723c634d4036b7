"""Timing helpers: clock sampling degrades gracefully without nvidia-smi; max over ranks."""
import multiprocessing as mp
import socket

from weightbridge_b200.utils.timing import ClockSampler, max_over_ranks


def test_clock_sampler_without_nvidia_smi(monkeypatch):
    import shutil
    monkeypatch.setattr(shutil, "which", lambda name: None)
    with ClockSampler() as c:
        pass
    s = c.summary()
    assert s["samples"] == 0 and s["reasons"] == ["unsampled"]


def test_clock_sampler_parses_csv(tmp_path):
    c = ClockSampler(raw_path=str(tmp_path / "raw.csv"))
    f = tmp_path / "clocks.csv"
    f.write_text("0, 1965, 1965, 800.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"
                 "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active\n"
                 "0, 300, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active\n")
    c._file = str(f)
    s = c.summary()
    assert s["samples"] == 3 and s["sm_max_mhz"] == 1965.0
    assert s["sm_mhz"] == 1882.5          # median of the samples under load (idle one dropped)
    assert s["reasons"] == ["sw_power_cap"]


def _rank(r, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=r, world_size=3)
    q.put(max_over_ranks(float(r * 10)))
    dist.destroy_process_group()


def test_max_over_ranks_gloo():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(3)]
    for p in ps:
        p.start()
    vals = [q.get(timeout=60) for _ in range(3)]
    for p in ps:
        p.join(10)
    assert vals == [20.0, 20.0, 20.0]
    assert max_over_ranks(3.5) == 3.5      # no process group: the value itself
