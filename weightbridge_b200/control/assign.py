"""Source assignment: which sender sends which entries to which receiver.

Senders whose shards of an entry are identical are replicas (trainer DP, or the dense part
of an EP-only layout); shards of different replica groups must not overlap.  For every
receiver entry and every replica group that overlaps it, one member of the group sends it.
Entries a single sender holds are fixed; replicated entries are then placed largest first on
the least-loaded member (ties: lowest rank), so every sender's NVLink egress carries about
the same bytes and the slowest link, which sets the sync time, is as short as possible.  When
the GPUs are known, a member on the receiver's own GPU is preferred (an HBM copy).

Parity: the reference deduplicates identical shards by keeping the lowest rank and raises
on partial overlap (``wbridge/backend/direct_sender.py:31-71``); the overlap rule is the
same, the choice among replicas is load-balanced instead of lowest-rank.
"""
from __future__ import annotations

import json
from collections import defaultdict

from ..core.shard import WeightData, box_copies


def _key(shards) -> str:
    return json.dumps(shards)


def replica_groups(sender_metas: list[WeightData]) -> dict[str, list[list[int]]]:
    """name -> list of replica groups (sender ranks with identical shards)."""
    out: dict[str, list[list[int]]] = {}
    by_name: dict[str, dict[str, list[int]]] = defaultdict(dict)
    for s, meta in enumerate(sender_metas):
        for name, shards, _ in meta:
            by_name[name].setdefault(_key(shards), []).append(s)
    for name, groups in by_name.items():
        glist = list(groups.values())
        keys = list(groups.keys())
        # different groups must not overlap
        for i in range(len(glist)):
            for j in range(i + 1, len(glist)):
                a = sender_metas[glist[i][0]].shards(name)
                b = sender_metas[glist[j][0]].shards(name)
                for sa in a:
                    for sb in b:
                        try:
                            bcs = box_copies(sa, sb)
                        except ValueError:
                            raise ValueError(f"senders {glist[i]} and {glist[j]} hold incompatible shards of {name!r}")
                        if bcs:
                            raise ValueError(
                                f"Partial shard overlap for {name!r} between sender ranks {glist[i][0]} and "
                                f"{glist[j][0]}: senders must have identical or non-overlapping shards")
        out[name] = glist
    return out


def _overlap_bytes(s_shards, r_shards, itemsize: int) -> int:
    n = 0
    for a in s_shards:
        for b in r_shards:
            n += sum(bc.numel for bc in box_copies(a, b))
    return n * itemsize


def overlap_sources(sender_metas: list[WeightData], receiver_metas: dict[int, WeightData]) -> dict[int, dict]:
    """For every receiver, the bytes of its entries by the senders that can serve them:
    ``{receiver: {(sender, ...): bytes}}``, a tuple of identical replicas (trainer DP, or a
    TP-replicated norm) or a single sender (its own shard).  The placement search's input."""
    groups = replica_groups(sender_metas)
    out: dict[int, dict] = {}
    for r, rmeta in receiver_metas.items():
        acc: dict[tuple, int] = defaultdict(int)
        for name, r_shards, r_dtype in rmeta:
            q = rmeta.quant(name)
            if q and q.get("role") == "scale":
                continue
            for group in groups.get(name, []):
                n = _overlap_bytes(sender_metas[group[0]].shards(name), r_shards, r_dtype.itemsize)
                if n:
                    acc[tuple(sorted(group))] += n
        out[r] = dict(acc)
    return out


def receiver_replicas(receiver_metas: dict[int, WeightData]) -> list[list[int]]:
    """Receivers with identical metadata (rollout replicas of one layout), groups of two or more."""
    by_key: dict[str, list[int]] = defaultdict(list)
    for r in sorted(receiver_metas):
        by_key[json.dumps(receiver_metas[r].to_jsonable(), sort_keys=True)].append(r)
    return [g for g in by_key.values() if len(g) > 1]


def assign_sources(sender_metas: list[WeightData], receiver_metas: dict[int, WeightData],
                   load_balance: bool = True, replica_consistent: bool = False,
                   sender_gpus: list | None = None, receiver_gpus: dict | None = None) -> dict[int, dict[int, list[str]]]:
    """``plan[sender][receiver] = [entry names]`` (both as indices into the inputs).

    Two passes: entries only one replica group can serve are assigned first (their load is
    fixed), then replicated entries, largest first, each to the least-loaded member of its
    group (longest-processing-time greedy), so every sender ends with about the same bytes.

    ``replica_consistent`` (multicast fan-out): receivers with identical metadata get each
    replicated entry from the same sender, so every sender writes the same entries to every
    replica of such a group and one multicast store can serve them all; the entry then costs
    its sender one copy of the bytes, not one per replica.

    ``sender_gpus`` / ``receiver_gpus`` (GPU identities, None for host memory): a replicated
    entry goes to a receiver from a member on the receiver's own GPU where there is one (an
    HBM copy, no link bytes, not counted as load); the others balance the link load.
    """
    def local(s_: int, r_: int) -> bool:
        """Sender ``s_`` and receiver ``r_`` share a GPU (the copy stays in its HBM)."""
        if sender_gpus is None or receiver_gpus is None:
            return False
        g = sender_gpus[s_]
        return g is not None and g == receiver_gpus.get(r_)

    groups = replica_groups(sender_metas)
    load = [0] * len(sender_metas)
    plan: dict[int, dict[int, list[str]]] = defaultdict(lambda: defaultdict(list))
    replicas = {r: [r] for r in receiver_metas}
    if replica_consistent:
        for g in receiver_replicas(receiver_metas):
            for r in g:
                replicas[r] = g
    flexible: list[tuple[int, int, str, list[int]]] = []      # (bytes, receiver, name, group)
    for r in sorted(receiver_metas):
        rmeta = receiver_metas[r]
        for name, r_shards, r_dtype in rmeta:
            q = rmeta.quant(name)
            if q and q.get("role") == "scale":
                continue
            for group in groups.get(name, []):
                s_shards = sender_metas[group[0]].shards(name)
                nbytes = _overlap_bytes(s_shards, r_shards, r_dtype.itemsize)
                if nbytes == 0:
                    continue
                if len(group) == 1 or not load_balance:
                    s = min(group)
                    load[s] += 0 if local(s, r) else nbytes
                    plan[s][r].append(name)
                elif replicas[r][0] == r:      # a replica group's entry is placed once, for all of it
                    flexible.append((nbytes, r, name, group))
    flexible.sort(key=lambda t: (-t[0], t[1], t[2]))
    for nbytes, r, name, group in flexible:
        near = [x for x in group if len(replicas[r]) == 1 and local(x, r)]
        if near:
            s = min(near, key=lambda x: (load[x], x))
        else:
            s = min(group, key=lambda x: (load[x], x))
            load[s] += nbytes
        for rr in replicas[r]:
            plan[s][rr].append(name)
    # keep each receiver's names in its metadata order (deterministic, cache friendly)
    order = {r: {n: i for i, n in enumerate(m.names())} for r, m in receiver_metas.items()}
    for s in plan:
        for r in plan[s]:
            plan[s][r].sort(key=lambda n: order[r][n])
    return {s: dict(v) for s, v in plan.items()}


def expected_senders(plan: dict[int, dict[int, list[str]]], receiver: int) -> list[int]:
    return sorted(s for s, rs in plan.items() if receiver in rs and rs[receiver])


def restrict(meta: WeightData, names) -> WeightData:
    keep = set(names)
    return WeightData({n: e for n, e in meta.to_jsonable().items() if n in keep})
