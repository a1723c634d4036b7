"""FSDP / DTensor trainer layout: HF-named parameters sharded along one dimension.

FSDP2 (``fully_shard``) keeps every parameter as a ``DTensor`` with placement ``Shard(0)``
over the data-parallel mesh; ``torch.chunk`` semantics decide the rows of each rank (chunks
of ``ceil(n / world)`` rows, trailing ranks possibly empty).  Each rank's local tensor is then
one box ``[(l, r, n), (0, d1, d1), ...]`` of the logical HF tensor, so a rank describes its
shard with no copy.  Shards are rarely aligned to the 128-row blocks of an fp8 rollout; the
senders of a split block exchange its amax (``core/splitq.py``).

The reference covers Megatron trainers only (``wbridge/utils/megatron_utils/qwen2.py``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Iterable

import torch

from ..core.shard import WeightData
from ..models.arch import ModelArch
from ..models.synthetic import synth_fill


def chunk_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows ``[l, r)`` of ``rank`` when ``n`` rows are split like ``torch.chunk(x, world)``."""
    c = -(-n // world) if n else 0
    l = min(rank * c, n)
    return l, min(l + c, n)


def shard_box(shape: tuple[int, ...], world: int, rank: int, dim: int = 0) -> list[tuple[int, int, int]] | None:
    """Box of ``rank``'s shard of a tensor of ``shape`` sharded on ``dim`` (None: empty shard);
    a tensor with fewer dimensions is sharded on dim 0."""
    box = [(0, d, d) for d in shape]
    if dim >= len(shape):
        dim = 0
    if world > 1 and shape:
        l, r = chunk_rows(shape[dim], world, rank)
        if l >= r:
            return None
        box[dim] = (l, r, shape[dim])
    return box


@dataclass
class FSDPLayout:
    """The shard of one data-parallel rank of an FSDP-sharded HF model."""
    arch: ModelArch
    world: int = 1
    rank: int = 0
    dim: int = 0

    def boxes(self) -> dict[str, list[tuple[int, int, int]]]:
        out = {}
        for name, shape in self.arch.hf_tensors():
            b = shard_box(shape, self.world, self.rank, self.dim)
            if b is not None:
                out[name] = b
        return out

    def param_shapes(self) -> dict[str, tuple[int, ...]]:
        return {n: tuple(r - l for l, r, _w in b) for n, b in self.boxes().items()}

    def allocate(self, device="cpu", dtype=torch.bfloat16, fill: bool = True, seed: int = 0) -> dict[str, torch.Tensor]:
        params = {n: torch.zeros(s, dtype=dtype, device=device) for n, s in self.param_shapes().items()}
        if fill:
            self.fill(params, seed)
        return params

    def fill(self, params: dict[str, torch.Tensor], seed: int = 0) -> None:
        for name, box in self.boxes().items():
            synth_fill(params[name], name, box, seed=seed)

    def to_wb(self, params: dict[str, torch.Tensor]) -> tuple[WeightData, dict[str, torch.Tensor]]:
        boxes = self.boxes()
        meta = {n: {"shard": boxes[n], "dtype": params[n].dtype} for n in boxes}
        return WeightData(meta), {n: params[n] for n in boxes}


def HFLayout(arch: ModelArch) -> FSDPLayout:
    """An unsharded HuggingFace model (trainer or rollout holding the plain HF state_dict,
    e.g. a transformers-based generator): every tensor whole, HF names."""
    return FSDPLayout(arch, world=1, rank=0)


def convert_to_wb(named_tensors: Iterable[tuple[str, Any]] | dict[str, Any]
                  ) -> tuple[WeightData, dict[str, torch.Tensor]]:
    """Metadata and local views of HF-named trainer tensors: ``DTensor``s with ``Shard(d)`` /
    ``Replicate`` placements on any number of mesh dimensions (FSDP2, HSDP, FSDP x TP,
    including FSDP's strided shards on top of TP), or plain tensors (the whole tensor)."""
    items = named_tensors.items() if isinstance(named_tensors, dict) else named_tensors
    meta, views = {}, {}
    for name, t in items:
        local, box = _local_and_box(t)
        if box is None:
            continue
        meta[name] = {"shard": box, "dtype": local.dtype}
        views[name] = local
    return WeightData(meta), views


def _local_and_box(t):
    """A DTensor's local tensor and its box.  Plain ``Shard(d)`` placements apply in
    mesh-dimension order, each cutting the current extent of tensor dim ``d`` like
    ``torch.chunk``; ``_StridedShard`` placements (FSDP2 on top of TP on the same dim) cut the
    chunk the plain shards left, after them.  HSDP is ``(Replicate(), Shard(0))``."""
    try:
        from torch.distributed.tensor import DTensor, Replicate, Shard
    except ImportError:              # torch without DTensor: plain tensors only
        DTensor = None
    if DTensor is None or not isinstance(t, DTensor):
        return t, [(0, d, d) for d in t.shape]
    mesh = t.device_mesh
    coord = mesh.get_coordinate()
    local = t.to_local()
    box = [[0, d, d] for d in t.shape]
    plain, strided = [], []
    for i, p in enumerate(t.placements):
        if isinstance(p, Replicate):
            continue
        if type(p) is Shard:
            plain.append((i, p))
        elif type(p).__name__ == "_StridedShard":
            strided.append((i, p))
        else:
            raise ValueError(f"unsupported placement {p} (Shard / Replicate / _StridedShard only)")
    for i, p in strided:
        inner = 1
        for j, q in plain:
            if q.dim == p.dim:
                inner *= mesh.size(j)
        if getattr(p, "split_factor", inner) != inner:
            raise ValueError(f"{p}: split factor {p.split_factor} is not the {inner} plain shards of dim {p.dim}")
    for i, p in plain + strided:
        l, r, w = box[p.dim]
        a, b = chunk_rows(r - l, mesh.size(i), coord[i])
        if a >= b:
            return local, None
        box[p.dim] = [l + a, l + b, w]
    box = [tuple(x) for x in box]
    if tuple(local.shape) != tuple(r - l for l, r, _w in box):
        raise ValueError(f"DTensor local shape {tuple(local.shape)} does not match its shard {box}")
    return local, box
