"""Where to put rollout workers that share the trainer's GPUs: the placement (worker -> GPU)
that minimises the busiest GPU's NVLink traffic of one sync.

Trainer rank s sits on GPU s.  A worker's bytes from a set of senders that can serve them (one
sender, or identical replicas) cost nothing on the links when one of those senders shares the
worker's GPU (an HBM copy); otherwise they leave the senders' GPUs (split evenly among the
replicas, as the load-balanced assignment roughly does) and enter the worker's GPU.  Up to 8
workers on up to 10 GPU slots every placement is tried; beyond that, hill climbing by swaps and
moves from the block and interleaved placements.
"""
from __future__ import annotations

import itertools
import math


def link_cost(placement: list[int], sources: dict[int, dict], n_gpus: int) -> float:
    """Busiest GPU's NVLink bytes (egress or ingress) for ``placement[w]`` = worker w's GPU."""
    egress = [0.0] * n_gpus
    ingress = [0.0] * n_gpus
    for w, g in enumerate(placement):
        for cands, b in sources[w].items():
            if g in cands:
                continue
            share = b / len(cands)
            for s in cands:
                egress[s] += share
            ingress[g] += b
    return max(max(egress), max(ingress))


def candidate_placements(n_workers: int, n_gpus: int, tp: int, replicas: int) -> dict[str, list[int]]:
    """The two structured placements: replicas in blocks, and replicas' ranks interleaved."""
    return {"block": [w % n_gpus for w in range(n_workers)],
            "interleaved": [((w % tp) * replicas + w // tp) % n_gpus for w in range(n_workers)]}


def best_placement(sources: dict[int, dict], n_gpus: int, tp: int, replicas: int) -> tuple[list[int], float]:
    """The placement with the least busiest-GPU traffic (ties: the first found), and its bytes."""
    n = len(sources)
    cap = max(1, math.ceil(n / n_gpus))
    slots = [g for g in range(n_gpus) for _ in range(cap)]
    starts = list(candidate_placements(n, n_gpus, tp, replicas).values())
    best = min(starts, key=lambda p: link_cost(p, sources, n_gpus))
    best_cost = link_cost(best, sources, n_gpus)
    if n <= 8 and len(slots) <= 10:
        for pick in itertools.permutations(range(len(slots)), n):
            p = [slots[i] for i in pick]
            c = link_cost(p, sources, n_gpus)
            if c < best_cost:
                best, best_cost = p, c
        return best, best_cost
    for start in starts:
        p, c = list(start), link_cost(start, sources, n_gpus)
        improved = True
        while improved:
            improved = False
            for i in range(n):
                moves = [("swap", j) for j in range(i + 1, n)]
                moves += [("move", g) for g in range(n_gpus) if p.count(g) < cap and g != p[i]]
                for kind, x in moves:
                    q = list(p)
                    if kind == "swap":
                        q[i], q[x] = q[x], q[i]
                    else:
                        q[i] = x
                    cq = link_cost(q, sources, n_gpus)
                    if cq < c:
                        p, c, improved = q, cq, True
        if c < best_cost:
            best, best_cost = p, c
    return best, best_cost
