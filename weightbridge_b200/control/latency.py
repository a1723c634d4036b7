"""Control-plane latency on this host: ``python -m weightbridge_b200.control.latency``.

Runs a rollout server (FastAPI controller + one receiver worker thread) and a sender in this
process with host tensors of a tiny model (``gpu_direct`` protocol through the C++ executor:
arm, ready / done handshakes, epoch flags), and reports per-sync medians: the whole
``send()``, the wait for the worker's ready key (the arm's round trip), the copy itself, and
``request_update`` on the worker side.  ``--direction push`` (the default here) measures the
protocol in which the sender copies; pulling, the worker copies and the sender waits for no
ready key.  The payload is ~8 MB, so the numbers are the control plane's own cost, the floor
under every sync's end-to-end time.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
import threading
import time


def measure(arm: str = "direct", syncs: int = 200, model: str = "tiny-llama", direction: str = "push") -> dict:
    import torch
    from ..models.arch import get_arch
    from ..parallel.megatron import MegatronLayout
    from ..parallel.sglang import SGLangLayout
    from ..utils.config import TransferConfig
    from .controller import WeightReceiverController
    from .receiver import WeightReceiver
    from .sender import WeightSender

    cfg = TransferConfig(mode="gpu_direct", arm=arm, connect_timeout_s=60, sync_timeout_s=60, direction=direction)
    arch = get_arch(model)
    rl = SGLangLayout(arch, tp=1)
    rparams = rl.allocate(dtype=torch.float32)
    rmeta, rviews = rl.to_wb(rparams)
    ctl = WeightReceiverController(worker_num=1, timeout_s=30)
    url = ctl.serve()
    recv = WeightReceiver(ctl.ipc_name, 0, rmeta, state_dict=rviews, config=cfg)
    sl = MegatronLayout(arch, tp=1)
    sparams = sl.allocate(dtype=torch.float32)
    smeta, sviews = sl.to_wb(sparams)
    sender = WeightSender("gpu_direct", [url], config=cfg)
    sender.connect(smeta)
    upd: list[float] = []
    stop = threading.Event()

    def worker():
        while not stop.is_set():
            t0 = time.perf_counter()
            if recv.request_update(timeout=1.0):
                upd.append((time.perf_counter() - t0) * 1e3)

    th = threading.Thread(target=worker, daemon=True)
    th.start()
    sends = []
    try:
        for _ in range(syncs):
            t0 = time.perf_counter()
            sender.send(sviews)
            sends.append((time.perf_counter() - t0) * 1e3)
    finally:
        stop.set()
        th.join(5)
        sender.disconnect()
        recv.stop()
        ctl.close()
    tail = slice(min(20, syncs // 4), None)             # drop the first syncs (plan compile, caches)
    hist = sender.history[tail]
    med = lambda xs: round(statistics.median(xs), 3) if xs else None   # noqa: E731
    return {"arm": arm, "direction": direction, "syncs": syncs, "model": model,
            "payload_bytes": hist[-1].bytes_written if hist else 0,
            "send_ms": med(sends[tail]), "wait_ready_ms": med([h.wait_ready_ms for h in hist]),
            "copy_ms": med([h.device_ms for h in hist]), "request_update_ms": med(upd[tail]),
            "note": "one process, host tensors; separate processes add socket hops but no GIL contention"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--arm", choices=["direct", "http"], default="direct")
    ap.add_argument("--syncs", type=int, default=200)
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--direction", choices=["push", "pull"], default="push")
    a = ap.parse_args(argv)
    print(json.dumps(measure(a.arm, a.syncs, a.model, a.direction)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
