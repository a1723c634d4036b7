"""The reference's data path re-expressed on torch.distributed, as a measured baseline.

Per (sender, receiver) pair: the sender packs every overlap box into one contiguous wire
buffer with one torch copy per box, ``isend``s it; the receiver ``irecv``s and unpacks with
one torch copy per box (``wbridge/utils/data.py:240-320``, ``wbridge/backend/direct_sender.py:
184-198``, ``wbridge/frontend/receiver.py:217-230``).  Unlike the shipped reference, the wire
buffer lives on the tensors' device, wire slices are typed, offsets are per tensor and only
overlapping pairs talk, so the algorithm actually runs; everything else (per-box copies,
NCCL point-to-point for the payload) is kept.  Source assignment uses the same replica
load balancing as the library so both paths move the same bytes.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..control.assign import assign_sources, restrict
from ..core.binding import Binding, pack_into, unpack_from
from ..core.shard import WeightData


@dataclass
class TorchP2PPlan:
    rank: int
    sends: dict[int, WeightData] = field(default_factory=dict)     # peer -> overlap (we send)
    recvs: dict[int, WeightData] = field(default_factory=dict)     # peer -> overlap (we receive)
    wires: dict[tuple[str, int], torch.Tensor] = field(default_factory=dict)

    @property
    def bytes_sent(self) -> int:
        return sum(o.total_nbytes() for o in self.sends.values())


def build_plan(rank: int, world: int, meta: WeightData, is_sender: bool, device, group=None) -> TorchP2PPlan:
    """Collective over ``group``: every rank contributes its metadata and role."""
    gathered = [None] * world
    dist.all_gather_object(gathered, (is_sender, meta.to_jsonable()), group=group)
    senders = [r for r, (s, _m) in enumerate(gathered) if s]
    receivers = [r for r, (s, _m) in enumerate(gathered) if not s]
    smetas = [WeightData(gathered[r][1]) for r in senders]
    rmetas = {r: WeightData(gathered[r][1]) for r in receivers}
    plan = assign_sources(smetas, rmetas)
    out = TorchP2PPlan(rank)
    for si, s in enumerate(senders):
        for r, names in plan.get(si, {}).items():
            ov = WeightData.compute_overlap(restrict(smetas[si], names), rmetas[r])
            if s == rank:
                out.sends[r] = ov
            if r == rank:
                out.recvs[s] = ov
    for peer, ov in out.sends.items():
        out.wires[("s", peer)] = torch.empty(ov.total_nbytes(), dtype=torch.uint8, device=device)
    for peer, ov in out.recvs.items():
        out.wires[("r", peer)] = torch.empty(ov.total_nbytes(), dtype=torch.uint8, device=device)
    return out


def sync(plan: TorchP2PPlan, binding: Binding, group=None) -> None:
    """One weight sync: pack + isend on senders, irecv + unpack on receivers."""
    works = []
    for peer, ov in plan.sends.items():
        wire = plan.wires[("s", peer)]
        pack_into(binding, ov, wire)
        works.append(dist.isend(wire, dst=peer, group=group))
    for peer in plan.recvs:
        works.append(dist.irecv(plan.wires[("r", peer)], src=peer, group=group))
    for w in works:
        w.wait()
    for peer, ov in plan.recvs.items():
        unpack_from(binding, ov, plan.wires[("r", peer)])
