"""Binding of ``WeightData`` entries to physical tensors, and the host-side pack/unpack.

A bound shard is a (possibly strided) tensor view whose shape is the shard's box extents.
Views let one logical entry live inside a fused buffer: the q rows of a grouped QKV weight
are ``qkv.view(G, (qpg + 2) * hd, H)[:, :qpg * hd]`` with box
``[(g0, g1, G), (0, qpg*hd, qpg*hd), (0, H, H)]``.  The reference required contiguous
per-entry tensors and rewrote the caller's dict (``wbridge/utils/data.py:219-238``); a
binding here leaves the caller's dict alone and accepts strided views.

``pack_into`` / ``unpack_from`` move overlap regions between bound tensors and a flat
wire buffer with torch strided copies.  They serve the reference-compatible
``WeightData.__call__`` API, the ``pack_for`` round trip and the tests' oracle; the
transfer engine uses the native executors instead.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from .shard import (Shard, WeightData, box_copies, contiguous_strides, shard_extents,
                    shard_numel)


@dataclass
class BoundShard:
    shard: Shard
    tensor: torch.Tensor          # view, shape == box extents
    strides: list[int]            # element strides per box dimension


@dataclass
class Binding:
    meta: WeightData
    entries: dict[str, list[BoundShard]] = field(default_factory=dict)
    device: torch.device = torch.device("cpu")

    def find(self, name: str, box: Shard):
        """(bound shard, BoxCopy) of the first local shard that fully contains ``box``."""
        found = self.find_all(name, box)
        if not found:
            raise ValueError(f"no local shard of {name} contains {box}")
        return found[0]

    def find_all(self, name: str, box: Shard) -> list:
        """Every (bound shard, BoxCopy) that fully contains ``box``: several when an entry's
        shards overlap (redundant expert slots, MLA's ``w_kc`` / ``w_vc`` inside ``kv_b_proj``)."""
        out = []
        for bs in self.entries[name]:
            try:
                bcs = box_copies(bs.shard, box, bs.strides, None)
            except ValueError:
                continue
            if len(bcs) == 1 and bcs[0].numel == shard_numel(box):
                out.append((bs, bcs[0]))
        return out


def _as_box_view(t: torch.Tensor, shard: Shard, name: str) -> BoundShard:
    ext = shard_extents(shard)
    if list(t.shape) == ext:
        return BoundShard(shard, t, list(t.stride()))
    if t.numel() != shard_numel(shard):
        raise ValueError(f"tensor for {name} has {t.numel()} elements, shard {shard} needs "
                         f"{shard_numel(shard)}")
    try:
        v = t.view(ext)
    except RuntimeError:
        raise ValueError(f"tensor for {name} (shape {tuple(t.shape)}, stride {t.stride()}) "
                         f"cannot be viewed as the shard box {ext}") from None
    return BoundShard(shard, v, list(v.stride()))


def bind(meta: WeightData, tensors: dict[str, Any]) -> Binding:
    """Bind every entry of ``meta`` to ``tensors[name]``.

    ``tensors[name]`` is a tensor (one shard: any shape viewable as the box; several
    shards: a contiguous buffer holding them back to back) or a list with one view per
    shard.  Tensors not named in ``meta`` are ignored.
    """
    b = Binding(meta)
    dev = None
    for name, shards, dtype in meta:
        if name not in tensors:
            raise KeyError(f"no tensor bound for entry {name!r}")
        t = tensors[name]
        views: list[BoundShard] = []
        if isinstance(t, (list, tuple)):
            if len(t) != len(shards):
                raise ValueError(f"{name}: {len(t)} views for {len(shards)} shards")
            views = [_as_box_view(v, s, name) for v, s in zip(t, shards)]
        elif len(shards) == 1:
            views = [_as_box_view(t, shards[0], name)]
        else:
            if not t.is_contiguous():
                raise ValueError(f"{name}: a multi-shard entry needs a contiguous buffer")
            flat = t.reshape(-1)
            off = 0
            for s in shards:
                n = shard_numel(s)
                views.append(_as_box_view(flat[off:off + n], s, name))
                off += n
            if off != flat.numel():
                raise ValueError(f"{name}: buffer has {flat.numel()} elements, shards need {off}")
        for v in views:
            if v.tensor.dtype != dtype:
                raise TypeError(f"{name}: tensor dtype {v.tensor.dtype} != metadata dtype {dtype}")
            dev = v.tensor.device if dev is None else dev
        b.entries[name] = views
    b.device = dev if dev is not None else torch.device("cpu")
    return b


def strided(t: torch.Tensor, offset: int, extents: Sequence[int], strides: Sequence[int]) -> torch.Tensor:
    """View of ``t``'s storage starting ``offset`` elements past ``t``'s first element."""
    return torch.as_strided(t, list(extents), list(strides), t.storage_offset() + offset)


def _region_views(binding: Binding, name: str, box: Shard, wire: torch.Tensor, bs=None):
    if bs is None:
        bs, _bc = binding.find(name, box)
    # wire side: the box packed contiguously; align its strides with the refinement
    bcs = box_copies(bs.shard, box, bs.strides, contiguous_strides(shard_extents(box)))
    assert len(bcs) == 1, (name, box)
    wire_bc = bcs[0]
    local = strided(bs.tensor, wire_bc.src_offset, wire_bc.extents, wire_bc.src_strides)
    packed = strided(wire, wire_bc.dst_offset, wire_bc.extents, wire_bc.dst_strides)
    return local, packed


def pack_into(binding: Binding, overlap: WeightData, out: torch.Tensor) -> None:
    """Gather ``overlap``'s regions of the bound tensors into ``out`` (flat uint8)."""
    from ..ops.quant_ref import block_quant_fp8_ref, convert_region
    starts = {name: start for start, _e, name, _s, _d in overlap.iter_with_intv()}
    for start, _end, name, shards, dtype in overlap.iter_with_intv():
        q = overlap.quant(name)
        if q and q.get("role") == "scale":
            continue                     # written together with its quantised weight
        off = start
        soff = starts.get(q["scale"]) if q else None
        for bi, box in enumerate(shards):
            n = shard_numel(box)
            seg = out[off:off + n * dtype.itemsize].view(dtype)
            local, packed = _region_views(binding, name, box, seg)
            if q:
                from .splitq import block_split, row_subregions
                if any(block_split([rows, cols], q["block"])[1] for _o, rows, cols in row_subregions(box)):
                    raise ValueError(f"{name}: region {box} cuts through {list(q['block'])} blocks; their "
                                     "scales need every sender's amax (WeightSender exchanges them)")
                qv, sv = block_quant_fp8_ref(local.reshape(shard_extents(box)), tuple(q["block"]))
                packed.copy_(qv.view(packed.shape))
                sbox = overlap.shards(q["scale"])[bi]
                ns = shard_numel(sbox)
                out[soff:soff + ns * 4].view(torch.float32).copy_(sv.reshape(-1))
                soff += ns * 4
            elif local.dtype == packed.dtype:
                packed.copy_(local)
            else:
                packed.copy_(convert_region(local, packed.dtype))
            off += n * dtype.itemsize


def unpack_from(binding: Binding, overlap: WeightData, chunk: torch.Tensor) -> None:
    """Scatter a packed ``chunk`` (``overlap`` layout) into the bound tensors: each region
    into every bound shard it intersects (an entry's shards may overlap, e.g. redundant
    expert slots, and the overlap then carries their shared elements once)."""
    chunk = chunk.reshape(-1).view(torch.uint8)
    if chunk.device != binding.device:
        chunk = chunk.to(binding.device)
    for start, _end, name, shards, dtype in overlap.iter_with_intv():
        off = start
        for box in shards:
            n = shard_numel(box)
            seg = chunk[off:off + n * dtype.itemsize].view(dtype)
            wire = contiguous_strides(shard_extents(box))
            wrote = 0
            for bs in binding.entries[name]:
                for bc in box_copies(box, bs.shard, wire, bs.strides):
                    strided(bs.tensor, bc.dst_offset, bc.extents, bc.dst_strides).copy_(
                        strided(seg, bc.src_offset, bc.extents, bc.src_strides))
                    wrote += bc.numel
            if wrote < n:
                raise ValueError(f"the local shards of {name} do not hold all of {box}")
            off += n * dtype.itemsize