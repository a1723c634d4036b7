"""Device timing and clock sampling for benchmarks and the per-sync stats record.

* ``EventTimer``: CUDA events on the launching stream; the elapsed device time of a region.
* ``max_over_ranks``: the slowest rank's value (a multi-GPU time is the max over ranks).
* ``ClockSampler``: ``nvidia-smi`` sampled every 200 ms in the background while a region
  runs; reports the median SM clock under load and the throttle reasons seen.
"""
from __future__ import annotations

import csv
import io
import os
import shutil
import signal
import statistics
import subprocess
import tempfile
import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


class EventTimer:
    def __init__(self, stream: torch.cuda.Stream | None = None):
        self.stream = stream
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        self.start.record(self.stream or torch.cuda.current_stream())
        return self

    def __exit__(self, *exc):
        self.end.record(self.stream or torch.cuda.current_stream())

    def ms(self) -> float:
        self.end.synchronize()
        return self.start.elapsed_time(self.end)


def max_over_ranks(value: float, group=None, device=None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    backend = dist.get_backend(group)
    dev = device if device is not None else (torch.device("cuda", torch.cuda.current_device())
                                             if backend == "nccl" else torch.device("cpu"))
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_COLS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


@dataclass
class ClockSampler:
    """Samples clocks of the visible GPUs with nvidia-smi while active (read-only)."""
    interval_ms: int = 200
    gpu_index: int | None = None
    raw_path: str | None = None
    _proc: subprocess.Popen | None = field(default=None, repr=False)
    _file: str | None = field(default=None, repr=False)

    def __enter__(self):
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        fd, self._file = tempfile.mkstemp(prefix="wb_clocks_", suffix=".csv")
        os.close(fd)
        cmd = [exe, f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.interval_ms}",
               f"--filename={self._file}"]
        if self.gpu_index is not None:
            cmd.insert(1, f"--id={self.gpu_index}")
        self._proc = subprocess.Popen(cmd, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL,
                                      start_new_session=True)
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self._proc is not None:
            time.sleep(0.25)
            try:
                os.killpg(self._proc.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
            self._proc.wait(timeout=10)

    def summary(self) -> dict:
        if not self._file or not os.path.exists(self._file):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        text = open(self._file).read()
        if self.raw_path:
            with open(self.raw_path, "w") as f:
                f.write(QUERY + "\n" + text)
        os.unlink(self._file)
        rows = [r for r in csv.reader(io.StringIO(text)) if len(r) >= 9]
        sm, smax, reasons = [], [], set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(REASON_COLS, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        hi = [x for x in sm if x >= 0.5 * max(sm)]
        return {"sm_mhz": statistics.median(hi), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}
