"""Full weight-sync benchmark: Megatron trainer layout -> SGLang rollout layout, synthetic
random-init weights of the named architecture, device-timed (CUDA events, max over ranks).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--model llama3-8b] [--impl wbridge|reference]

Layout per N (strong scaling: the model, hence the bytes moved per sync, is fixed):
  N=1  colocated: trainer TP1 and rollout TP1 on the same GPU (HBM -> HBM)
  N=2  TP1 -> TP1, trainer GPU 0, rollout GPU 1 (NVLink)
  N=4  TP2 -> TP2, trainer GPUs 0-1, rollout GPUs 2-3
  N=8  TP4 -> TP4, trainer GPUs 0-3, rollout GPUs 4-7
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "full weight-sync latency (s, device-timed, max over ranks) + effective GB/s/GPU"
BASELINE_PUBLISHED = None   # the reference publishes no number


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--impl", default="wbridge", choices=["wbridge", "reference"])
    p.add_argument("--mode", type=int, default=None, help="kernel mode (0 vector, 1/2/3 TMA bulk)")
    p.add_argument("--piece", type=int, default=None)
    p.add_argument("--item-bytes", type=int, default=1 << 19)
    p.add_argument("--no-verify", action="store_true")
    return p.parse_args()


def reference_unavailable(args):
    why = ("the reference's stock send path cannot run: WeightTensorBridge binds uint8 wire slices and "
           "then asserts they match the bf16 metadata dtype (wbridge/utils/data.py:227-229, 300-305), and "
           "GPUDirectSender NCCL-sends a CPU pack buffer (data.py:300, direct_sender.py:192-195)")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


def colocated_one_gpu(args):
    from weightbridge_b200.core.binding import bind
    from weightbridge_b200.core.plan import lower_ops, phys_binding, plan_pair
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.ops.executor import LaunchConfig, TransferProgram
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from weightbridge_b200.parallel.sglang import SGLangLayout
    from weightbridge_b200.utils.timing import ClockSampler, EventTimer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    arch = get_arch(args.model)
    meg = MegatronLayout(arch, tp=1)
    sgl = SGLangLayout(arch, tp=1)
    t0 = time.time()
    sparams = meg.allocate(device=dev, dtype=torch.bfloat16)
    smeta, sviews = meg.to_wb(sparams)
    rparams = sgl.allocate(device=dev, dtype=torch.bfloat16)
    rmeta, rviews = sgl.to_wb(rparams)
    ops = plan_pair(phys_binding(bind(smeta, sviews)), phys_binding(bind(rmeta, rviews)))
    tables = lower_ops(ops, lambda a: 0, lambda a: 0, item_bytes=args.item_bytes)
    cfg = LaunchConfig.from_env()
    if args.mode is not None:
        cfg.mode = args.mode
    if args.piece is not None:
        cfg.piece_bytes = args.piece
    flag = torch.zeros(1, dtype=torch.int64, device=dev)
    prog = TransferProgram(tables, dev, [flag.data_ptr()], cfg)
    setup_s = time.time() - t0
    stream = torch.cuda.Stream(dev)
    for w in range(args.warmup):
        prog.launch(epoch=w + 1, stream=stream)
    torch.cuda.synchronize()
    with ClockSampler(gpu_index=None) as clk:
        torch.cuda.synchronize()
        with EventTimer(stream) as tm:
            for k in range(args.steps):
                prog.launch(epoch=args.warmup + k + 1, stream=stream)
        ms = tm.ms() / args.steps
        torch.cuda.synchronize()
    status = prog.read_status()
    ok = None
    if not args.no_verify:
        expected = sgl.allocate(device=dev, dtype=torch.bfloat16, fill=True)
        ok = all(torch.equal(rparams[n], expected[n]) for n in rparams)
        del expected
    payload = tables.bytes_written
    lat = ms / 1e3
    gbs = payload / lat / 1e9
    return {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) weights, hashed per element)",
        "config": {"model": args.model, "layout": "Megatron TP1 -> SGLang TP1, colocated on one GPU",
                   "global_batch": None, "seq_len": None, "parallelism": "tp1->tp1",
                   "payload_bytes": payload, "l2": "inputs larger than L2 (16 GB per sync)",
                   "kernel_mode": cfg.mode, "piece_bytes": cfg.piece_bytes, "items": len(tables.items),
                   "grid": prog.grid(), "path": "in-process data plane"},
        "latency_s": round(lat, 6), "gbs_per_gpu": round(gbs, 2),
        "hbm_traffic_gbs": round(2 * payload / lat / 1e9, 1),
        "clocks": clk.summary(), "gpu_launches": args.steps, "status": status, "verified": ok,
        "setup_s": round(setup_s, 1),
    }


def main():
    args = parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return
    if args.gpus != 1:
        raise SystemExit("multi-GPU bench arrives with the IPC control plane")
    res = colocated_one_gpu(args)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
