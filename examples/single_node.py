"""Single-node example of the public API: a Megatron-layout trainer pushes its weights into
an SGLang-layout rollout engine after every "training step".

Process layout (the shape of a real RL job, without Ray):

    rollout engine  (FastAPI + WeightReceiverController, hosts the HTTP control plane)
    ├── worker 0 .. M-1  (child processes, like SGLang schedulers: each owns its parameters,
    │                     runs a WeightReceiver and calls request_update between batches)
    trainer rank 0 .. N-1 (torch.distributed group; WeightSender.connect once, send per step)

    python examples/single_node.py --device cpu                 # gloo payload path, any machine
    python examples/single_node.py --device cuda                # CUDA IPC + sm_100a kernel, colocated on GPU 0
    python examples/single_node.py --device cuda --disaggregated  # trainers and workers on different GPUs
    python examples/single_node.py --trainer fsdp --trainers 3    # an FSDP-sharded trainer instead

Weights are synthetic (the tiny Llama-style model by default); every worker checks after
each update that it holds exactly the trainer's weights of that step.
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


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]

def share_cores(args) -> None:
    """All the example's processes run on this host: split the cores between their intra-op
    thread pools instead of letting every process start one thread per core."""
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // (args.trainers + args.workers + 1)))



def device_for(args, role: str, rank: int) -> str:
    if args.device == "cpu":
        return "cpu"
    if not args.disaggregated:
        return "cuda:0"
    return f"cuda:{rank}" if role == "trainer" else f"cuda:{args.trainers + rank}"


# -- rollout side --------------------------------------------------------------------------
def worker(args, ipc_name: str, rank: int, results):
    share_cores(args)
    """One rollout worker: owns its shard of the SGLang parameters, takes updates."""
    from weightbridge_b200 import SGLangLayout, TransferConfig, WeightReceiver
    from weightbridge_b200.models.arch import get_arch
    dev = device_for(args, "rollout", rank)
    if dev != "cpu":
        torch.cuda.set_device(torch.device(dev))
    lay = SGLangLayout(get_arch(args.model), tp=args.workers, tp_rank=rank)
    params = lay.allocate(device=dev, dtype=args.dtype)
    meta, views = lay.to_wb(params)
    cfg = TransferConfig(mode=args.mode)
    receiver = WeightReceiver(ipc_name, rank, meta, state_dict=views, config=cfg)
    for step in range(args.steps):
        # a scheduler would serve batches here and call request_update between two of them
        if not receiver.request_update(timeout=120):
            results.put(("worker", rank, step, False))
            break
        expected = lay.allocate(device=dev, dtype=args.dtype, fill=True, seed=step)
        ok = all(torch.equal(params[n], expected[n]) for n in params)
        results.put(("worker", rank, step, ok))
    receiver.stop()


def rollout_engine(args, port: int, results):
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import WeightReceiverController
    app = FastAPI()
    controller = WeightReceiverController(app)
    ctx = mp.get_context("spawn")
    workers = [ctx.Process(target=worker, args=(args, controller.ipc_name, r, results)) for r in range(args.workers)]
    for p in workers:
        p.start()
    controller.set_worker_num(args.workers)
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    threading.Thread(target=server.run, daemon=True).start()
    for p in workers:
        p.join()
    server.should_exit = True
    controller.close()


# -- trainer side --------------------------------------------------------------------------
def trainer(args, rank: int, dist_port: int, url: str, results):
    share_cores(args)
    import torch.distributed as dist
    from weightbridge_b200 import MegatronLayout, TransferConfig, WeightSender
    from weightbridge_b200.models.arch import get_arch
    dev = device_for(args, "trainer", rank)
    if dev != "cpu":
        torch.cuda.set_device(torch.device(dev))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{dist_port}", rank=rank,
                            world_size=args.trainers)
    if args.trainer == "fsdp":              # FSDP2 / DTensor trainer: Shard(0) rows per rank
        from weightbridge_b200 import FSDPLayout
        lay = FSDPLayout(get_arch(args.model), world=args.trainers, rank=rank)
    else:
        lay = MegatronLayout(get_arch(args.model), tp=args.trainers, tp_rank=rank)
    params = lay.allocate(device=dev, dtype=args.dtype, seed=0)
    meta, views = lay.to_wb(params)          # HF-named boxes bound to views of the params
    sender = WeightSender(args.mode, [url], config=TransferConfig(mode=args.mode))
    sender.connect(meta)
    for step in range(args.steps):
        if step:
            lay.fill(params, seed=step)      # stands in for an optimizer step
        stats = sender.send(views)
        results.put(("trainer", rank, step, stats.device_ms))
    sender.disconnect()
    dist.destroy_process_group()


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--device", default="cpu", choices=["cpu", "cuda"])
    p.add_argument("--disaggregated", action="store_true")
    p.add_argument("--model", default="tiny-llama")
    p.add_argument("--trainers", type=int, default=2)
    p.add_argument("--trainer", default="megatron", choices=["megatron", "fsdp"],
                   help="trainer layout: Megatron TP over the trainer ranks, or FSDP rows")
    p.add_argument("--workers", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    args = p.parse_args(argv)
    args.mode = "cpu_direct" if args.device == "cpu" else "gpu_direct"
    args.dtype = torch.float32 if args.device == "cpu" else torch.bfloat16
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port, dist_port = free_port(), free_port()
    url = f"http://127.0.0.1:{port}"
    procs = [ctx.Process(target=rollout_engine, args=(args, port, results))]
    procs += [ctx.Process(target=trainer, args=(args, r, dist_port, url, results)) for r in range(args.trainers)]
    for pr in procs:
        pr.start()
    want = args.steps * (args.workers + args.trainers)
    got, deadline = [], time.time() + 600
    while len(got) < want and time.time() < deadline:
        try:
            got.append(results.get(timeout=1))
        except queue.Empty:
            if any(pr.exitcode not in (None, 0) for pr in procs):
                break
    for pr in procs:
        pr.join(timeout=30)
        if pr.is_alive():
            pr.kill()
    checks = [g for g in got if g[0] == "worker"]
    ok = len(checks) == args.steps * args.workers and all(g[3] for g in checks)
    for g in sorted(got):
        print(g)
    print("all syncs verified" if ok else "FAILED")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
