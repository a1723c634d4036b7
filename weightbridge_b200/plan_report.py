"""Dry-run planner: what a sync between two layouts moves, without allocating a byte.

    python -m weightbridge_b200.plan_report --model qwen3-30b-a3b --trainer ep=4 \\
        --rollout tp=4,moe_ep=4,quant=fp8_experts
    python -m weightbridge_b200.plan_report --model llama3-8b --trainer tp=2,pp=2 --rollout tp=1 --replicas 4 --json
    python -m weightbridge_b200.plan_report --model llama3-8b --trainer tp=1 --rollout tp=1 --replicas 7 --multicast
    python -m weightbridge_b200.plan_report --model llama3-70b --trainer tp=8 --rollout tp=4 --replicas 2 --colocated interleaved

Builds both layouts on the ``meta`` device, runs the source assignment and the planner for
every (sender, receiver) pair, and reports per-sender and per-receiver bytes, work rows,
quantised blocks and split-block pieces, plus the sync time the busiest link allows
(``--multicast``: the ``nvls`` mode's plan, multicast copies counted once per replica group).  Trainer
ranks are enumerated as data-parallel replica x pipeline stage x expert-parallel rank x max(tp, etp) with
``tp_rank = t % tp`` and ``etp_rank = t % etp`` (``--trainer-kind fsdp``: ``world`` ranks of
an FSDP-sharded model); rollout workers as replica x tp rank.
The reference has no equivalent (it plans inside ``connect``, ``wbridge/backend/direct_sender.py:74-168``).
"""
from __future__ import annotations

import argparse
import json
import sys

import torch

from .control.assign import assign_sources
from .core.binding import bind
from .core.plan import lower_ops, phys_binding, plan_pair
from .models.arch import get_arch
from .parallel.megatron import MegatronLayout
from .parallel.sglang import SGLangLayout

_ABS = lambda _alloc: 0      # noqa: E731  (meta tensors: every address is 0)


def _kv(spec: str) -> dict:
    out: dict = {}
    for part in filter(None, (p.strip() for p in spec.split(","))):
        k, _, v = part.partition("=")
        out[k] = int(v) if v.lstrip("-").isdigit() else (None if v in ("", "none") else v)
    return out


def trainer_layouts(arch, spec: dict, kind: str = "megatron") -> list:
    if kind == "fsdp":
        from .parallel.fsdp import FSDPLayout
        world = int(spec.get("world", 1))
        return [FSDPLayout(arch, world=world, rank=i, dim=int(spec.get("dim", 0))) for i in range(world)]
    tp, pp, ep, etp, dp = (int(spec.get(k, 1)) for k in ("tp", "pp", "ep", "etp", "dp"))
    extra = {k: v for k, v in spec.items() if k not in ("tp", "pp", "ep", "etp", "dp")}
    return [MegatronLayout(arch, tp=tp, pp=pp, ep=ep, etp=etp, tp_rank=t % tp, pp_rank=p, ep_rank=e,
                           etp_rank=t % etp, **extra)
            for _d in range(dp) for p in range(pp) for e in range(ep) for t in range(max(tp, etp))]


def rollout_layouts(arch, spec: dict, replicas: int) -> list[SGLangLayout]:
    tp = int(spec.get("tp", 1))
    extra = {k: v for k, v in spec.items() if k != "tp"}
    return [SGLangLayout(arch, tp=tp, tp_rank=t, **extra) for _ in range(replicas) for t in range(tp)]


def _meta_binding(lay):
    params = lay.allocate(device="meta", dtype=torch.bfloat16, fill=False)
    meta, views = lay.to_wb(params)
    return meta, phys_binding(bind(meta, views))


def report(model: str, trainer: dict, rollout: dict, replicas: int = 1, link_gbs: float | None = None,
           trainer_kind: str = "megatron", multicast: bool = False, mc_gbs: float | None = None,
           colocated: str | bool = False) -> dict:
    """``link_gbs``: per-GPU link bandwidth of the estimate (default: the measured GPU -> GPU
    peak, ``ops/microbench.py:peer_peak``).  ``multicast``: the ``nvls`` mode's plan, where the
    workers with identical layouts (replicas) form groups, the source assignment is
    replica-consistent and a sender's aligned same-dtype copies leave its GPU once per group,
    at ``mc_gbs`` (default: the measured multicast store rate, ``--case mc-peak``).
    GPUs: trainer rank s on GPU s; rollout worker w (tp rank t of replica e) on GPU ``trainers + w``,
    or beside the trainer ranks with ``colocated``: ``"block"`` (or True) puts it on GPU
    ``w % trainers`` (replica after replica), ``"interleaved"`` on GPU ``(t * replicas + e) %
    trainers`` (the replicas' ranks alternate), ``"best"`` where the placement search puts it
    (``utils/placement.py``); bytes between a trainer rank and a worker on its own GPU stay in
    HBM."""
    from .utils.links import busiest_link, link_bytes
    from .control.assign import receiver_replicas
    from .core.plan import multicast_ok
    from .ops.microbench import _mc_peak_gbs, _peer_peak_gbs
    if link_gbs is None:
        link_gbs = _peer_peak_gbs()
    if mc_gbs is None:
        mc_gbs = (_mc_peak_gbs() or link_gbs) if multicast else link_gbs
    arch = get_arch(model)
    senders = [_meta_binding(l) for l in trainer_layouts(arch, trainer, trainer_kind)]
    receivers = [_meta_binding(l) for l in rollout_layouts(arch, rollout, replicas)]
    smetas = [m for m, _ in senders]
    rmetas = {r: m for r, (m, _) in enumerate(receivers)}
    ntp = int(rollout.get("tp", 1))
    placement = None
    if colocated == "best":                 # search the worker -> GPU placement (utils/placement.py)
        from .control.assign import overlap_sources
        from .utils.placement import best_placement
        placement, _cost = best_placement(overlap_sources(smetas, rmetas), len(senders), ntp, replicas)
        gpu = placement.__getitem__
    elif colocated == "interleaved":
        gpu = lambda w: ((w % ntp) * replicas + w // ntp) % len(senders)       # noqa: E731
    elif colocated:
        gpu = lambda w: w % len(senders)                                          # noqa: E731
    else:
        gpu = lambda w: len(senders) + w                                          # noqa: E731
    # the assignment the sender's connect makes: GPU-aware (a replicated entry from the worker's
    # own GPU where a trainer rank there holds it), replica-consistent with multicast
    plan = assign_sources(smetas, rmetas, replica_consistent=multicast, sender_gpus=list(range(len(senders))),
                          receiver_gpus={w: gpu(w) for w in rmetas})
    groups = {g[0]: g for g in receiver_replicas(rmetas)} if multicast else {}
    grouped = {r for g in groups.values() for r in g}
    routes: list[dict] = []
    srows, ingress = [], [0] * len(receivers)
    for s, (smeta, sphys) in enumerate(senders):
        row = {"sender": s, "targets": 0, "bytes_read": 0, "bytes_written": 0, "items": 0,
               "quant_blocks": 0, "split_pieces": 0, "multicast_bytes": 0}
        for r, names in sorted(plan.get(s, {}).items()):
            if not names or (r in grouped and r not in groups):
                continue                       # a replica group is planned through its first worker
            ops = plan_pair(sphys, receivers[r][1], names=names)
            reps = groups.get(r, [r])
            parts = [(lower_ops(ops, _ABS, _ABS, receiver=r), len(reps))]
            if len(reps) > 1:                  # multicast copies once, the rest once per replica
                mc = [o for o in ops if multicast_ok(o, _ABS, _ABS)]
                uni = [o for o in ops if not multicast_ok(o, _ABS, _ABS)]
                mct = lower_ops(mc, _ABS, _ABS, multicast=True)
                row["multicast_bytes"] += mct.bytes_written
                parts = [(mct, 0), (lower_ops(uni, _ABS, _ABS, receiver=r), len(reps))]
            for t, copies in parts:
                row["bytes_read"] += t.bytes_read
                row["bytes_written"] += t.bytes_written * copies
                row["items"] += len(t.items)
                row["quant_blocks"] += len(t.qwork) * max(copies, 1)
                row["split_pieces"] += len(t.pieces) * max(copies, 1)
                for rr in reps:
                    ingress[rr] += t.bytes_written
                if copies == 0:
                    routes.append({"src": s, "dst": [gpu(rr) for rr in reps], "bytes": t.bytes_written,
                                   "multicast": True})
                else:
                    routes += [{"src": s, "dst": [gpu(rr)], "bytes": t.bytes_written, "multicast": False}
                               for rr in reps]
            row["targets"] += len(reps)
        srows.append(row)
    # time per GPU: unicast bytes at the peer rate, multicast bytes at the multicast rate;
    # bytes between a trainer rank and a worker on its own GPU stay in HBM
    egress_b, mc_b, ingress_b, local = link_bytes(routes)
    worst = busiest_link(routes, link_gbs, mc_gbs)
    egress = max((r["bytes_written"] for r in srows), default=0)
    inmax = max(ingress, default=0)
    return {
        "model": model, "trainer_kind": trainer_kind, "trainer": trainer, "rollout": rollout, "replicas": replicas,
        "multicast": multicast,
        "senders": srows,
        "receivers": [{"receiver": r, "ingress_bytes": b,
                       "senders": sorted(s for s, t in plan.items() if t.get(r))} for r, b in enumerate(ingress)],
        "total_written_bytes": sum(ingress),
        "busiest_sender_bytes": egress, "busiest_receiver_bytes": inmax,
        "link_gbs": link_gbs, "multicast_gbs": mc_gbs if multicast else None,
        "colocated": colocated, "placement": placement if placement is not None else
        ([gpu(w) for w in range(len(receivers))] if colocated else None), "gpu_local_bytes": local,
        "gpu_egress_bytes": {str(d): b for d, b in sorted(egress_b.items())},
        "gpu_multicast_egress_bytes": {str(d): b for d, b in sorted(mc_b.items())},
        "gpu_ingress_bytes": {str(d): b for d, b in sorted(ingress_b.items())},
        "busiest_gpu": None if worst is None else {"side": worst[0], "gpu": worst[1]},
        "link_bound_ms": 0.0 if worst is None else worst[2],
        "note": "NVLink-bound estimate (the busiest GPU's egress or ingress); bytes between a trainer rank "
                "and a worker on its own GPU move through HBM and are left out",
    }


def _gb(n: int) -> str:
    return f"{n / 1e9:.3f}"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True)
    ap.add_argument("--trainer", default="", help="Megatron layout, e.g. tp=2,pp=2 or ep=4,etp=2; FSDP: world=8")
    ap.add_argument("--trainer-kind", default="megatron", choices=["megatron", "fsdp"])
    ap.add_argument("--rollout", default="", help="SGLang layout, e.g. tp=4,moe_ep=4,quant=fp8_experts")
    ap.add_argument("--replicas", type=int, default=1, help="rollout replicas (each with the rollout layout)")
    ap.add_argument("--link-gbs", type=float, default=None,
                    help="per-GPU link bandwidth for the estimate (default: the measured peer peak)")
    ap.add_argument("--multicast", action="store_true",
                    help="the nvls mode: replicas of one layout served by multicast stores")
    ap.add_argument("--mc-gbs", type=float, default=None,
                    help="multicast store rate out of one GPU (default: the measured one)")
    ap.add_argument("--colocated", nargs="?", const="block", default=None, choices=["block", "interleaved", "best"],
                    help="rollout workers on the trainers' GPUs: block (worker w on GPU w %% trainers), "
                         "interleaved (tp rank t of replica e on GPU t * replicas + e) or best (searched); "
                         "else GPUs of their own")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    rep = report(a.model, _kv(a.trainer), _kv(a.rollout), a.replicas, a.link_gbs, a.trainer_kind,
                 multicast=a.multicast, mc_gbs=a.mc_gbs, colocated=a.colocated or False)
    if a.json:
        print(json.dumps(rep))
        return 0
    print(f"{a.model}: trainer {a.trainer or 'tp=1'} ({len(rep['senders'])} ranks) -> rollout "
          f"{a.rollout or 'tp=1'} x{a.replicas} ({len(rep['receivers'])} workers)")
    print(f"{'sender':>6} {'targets':>7} {'read GB':>9} {'written GB':>10} {'multicast GB':>12} {'items':>8} "
          f"{'quant blk':>9} {'split pcs':>9}")
    for r in rep["senders"]:
        print(f"{r['sender']:>6} {r['targets']:>7} {_gb(r['bytes_read']):>9} {_gb(r['bytes_written']):>10} "
              f"{_gb(r['multicast_bytes']):>12} {r['items']:>8} {r['quant_blocks']:>9} {r['split_pieces']:>9}")
    print(f"{'worker':>6} {'ingress GB':>10}  senders")
    for r in rep["receivers"]:
        print(f"{r['receiver']:>6} {_gb(r['ingress_bytes']):>10}  {r['senders']}")
    mc = max((r["multicast_bytes"] for r in rep["senders"]), default=0)
    line = f"total written {_gb(rep['total_written_bytes'])} GB; busiest sender {_gb(rep['busiest_sender_bytes'])} GB"
    if rep["multicast"]:
        line += f" unicast + {_gb(mc)} GB multicast"
    line += f", busiest worker {_gb(rep['busiest_receiver_bytes'])} GB"
    if rep["colocated"]:
        line += f"; {_gb(rep['gpu_local_bytes'])} GB stay within GPUs (worker -> GPU {rep['placement']})"
    worst = rep["busiest_gpu"]
    where = f" ({worst['side']} of GPU {worst['gpu']})" if worst else ""
    line += f" -> {rep['link_bound_ms']:.2f} ms{where} at {rep['link_gbs']:.0f} GB/s per link"
    if rep["multicast"]:
        line += f", multicast at {rep['multicast_gbs']:.0f} GB/s"
    print(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
