"""Hand-built shard metadata through the public API, without any layout adapter.

The scenario of the reference's example (``examples/train.py:21-31, 71-117`` there): two
trainer ranks and a rollout engine with two workers, three float32 tensors of shape [4, 8]:

    uneven_weight  rows split unevenly:  rank 0 holds rows [0, 1), rank 1 rows [1, 4)
    col_weight     columns split:        rank 0 holds cols [0, 4), rank 1 cols [4, 8)
    dup_weight     duplicated:           both ranks hold the whole tensor (one of them sends it)

and every rollout worker holds one half of the rows of all three.  Worker tensors are plain
flat buffers, as in the reference (any shape with the box's element count binds), and are
handed over at ``request_update`` (the reference's receiver flow).

    python examples/raw_shards.py --device cpu      # cpu_direct: C++ pack/unpack + gloo
    python examples/raw_shards.py --device cuda     # gpu_direct: CUDA IPC + sm_100a kernel on GPU 0

The reference orchestrates the same processes with Ray placement groups; here plain
``multiprocessing`` does it, so the example runs on one machine with nothing else installed.
"""
from __future__ import annotations

import argparse
import multiprocessing as mp
import os
import queue
import socket
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

ROWS, COLS = 4, 8
NAMES = ("uneven_weight", "col_weight", "dup_weight")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]

def share_cores(args) -> None:
    """All the example's processes run on this host: split the cores between their intra-op
    thread pools instead of letting every process start one thread per core."""
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // (5)))



def full_tensor(name: str, step: int) -> torch.Tensor:
    """The logical [4, 8] tensor of ``name`` after training step ``step``."""
    base = {"uneven_weight": 0.0, "col_weight": 100.0, "dup_weight": 200.0}[name]
    return torch.arange(ROWS * COLS, dtype=torch.float32).view(ROWS, COLS) + base + 1000.0 * step


def sender_meta(rank: int):
    from weightbridge_b200 import WeightData
    rows = [(0, 1, ROWS), (1, ROWS, ROWS)][rank]
    cols = [(0, COLS // 2, COLS), (COLS // 2, COLS, COLS)][rank]
    return WeightData({
        "uneven_weight": {"shard": [rows, (0, COLS, COLS)], "dtype": torch.float32},
        "col_weight": {"shard": [(0, ROWS, ROWS), cols], "dtype": torch.float32},
        "dup_weight": {"shard": [(0, ROWS, ROWS), (0, COLS, COLS)], "dtype": torch.float32},
    })


def receiver_meta(rank: int):
    from weightbridge_b200 import WeightData
    half = ROWS // 2
    box = [(rank * half, (rank + 1) * half, ROWS), (0, COLS, COLS)]
    return WeightData({n: {"shard": box, "dtype": torch.float32} for n in NAMES})


def local_slice(t: torch.Tensor, box) -> torch.Tensor:
    return t[tuple(slice(l, r) for l, r, _w in box)]


# -- rollout side --------------------------------------------------------------------------
def worker(args, ipc_name: str, rank: int, results):
    share_cores(args)
    from weightbridge_b200 import TransferConfig, WeightReceiver
    from weightbridge_b200.core.shard import shard_numel
    dev = "cpu" if args.device == "cpu" else "cuda:0"
    meta = receiver_meta(rank)
    # flat buffers, one per name, allocated by the "engine"
    bufs = {n: torch.zeros(shard_numel(meta.shards(n)[0]), dtype=torch.float32, device=dev) for n in NAMES}
    recv = WeightReceiver(ipc_name, rank, meta, device=dev, config=TransferConfig(mode=args.mode))
    ok = True
    try:
        for step in range(args.steps):
            deadline = time.time() + 60
            while not recv.request_update(bufs, timeout=1.0):      # between two "batches"
                if time.time() > deadline:
                    raise TimeoutError("no weights arrived")
            for n in NAMES:
                exp = local_slice(full_tensor(n, step), meta.shards(n)[0]).reshape(-1)
                if not torch.equal(bufs[n].cpu(), exp):
                    ok = False
                    print(f"[worker {rank}] step {step}: {n} differs", flush=True)
    except Exception as e:  # reported to the parent
        ok = False
        print(f"[worker {rank}] {type(e).__name__}: {e}", flush=True)
    finally:
        recv.stop()
    results.put(("worker", rank, ok))


def rollout_engine(args, port: int, results, ready):
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import WeightReceiverController
    app = FastAPI()
    ctl = WeightReceiverController(app, worker_num=2, timeout_s=60)
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=worker, args=(args, ctl.ipc_name, r, results)) for r in range(2)]
    for p in procs:
        p.start()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    while not server.started:
        time.sleep(0.05)
    ready.put(True)
    for p in procs:
        p.join(300)
    server.should_exit = True
    th.join(10)
    ctl.close()


# -- trainer side --------------------------------------------------------------------------
def trainer(args, rank: int, dist_port: int, url: str, results):
    share_cores(args)
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{dist_port}", rank=rank, world_size=2)
    dev = "cpu" if args.device == "cpu" else "cuda:0"
    if dev != "cpu":
        torch.cuda.set_device(0)
    meta = sender_meta(rank)
    params = {n: local_slice(full_tensor(n, 0), meta.shards(n)[0]).contiguous().to(dev) for n in NAMES}
    sender = WeightSender(args.mode, [url], config=TransferConfig(mode=args.mode))
    sender.connect(meta)
    for step in range(args.steps):
        for n in NAMES:                    # the "optimizer step": new values in place
            params[n].copy_(local_slice(full_tensor(n, step), meta.shards(n)[0]))
        sender.send(params)
    sender.disconnect()
    dist.destroy_process_group()
    results.put(("trainer", rank, True))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--steps", type=int, default=3)
    args = ap.parse_args(argv)
    args.mode = "cpu_direct" if args.device == "cpu" else "gpu_direct"
    ctx = mp.get_context("spawn")
    results, ready = ctx.Queue(), ctx.Queue()
    port, dist_port = free_port(), free_port()
    engine = ctx.Process(target=rollout_engine, args=(args, port, results, ready))
    engine.start()
    ready.get(timeout=120)
    url = f"http://127.0.0.1:{port}"
    trainers = [ctx.Process(target=trainer, args=(args, r, dist_port, url, results)) for r in range(2)]
    for p in trainers:
        p.start()
    got = []
    try:
        while len(got) < 4:
            got.append(results.get(timeout=300))
    except queue.Empty:
        print("timed out waiting for the processes", flush=True)
    for p in trainers + [engine]:
        p.join(30)
        if p.is_alive():
            p.kill()
    ok = len(got) == 4 and all(r[2] for r in got)
    print(f"{'OK' if ok else 'FAILED'}: {sorted(got)}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
