"""Shard algebra: N-d boxes inside logical (HF-named) tensors, their alignment and overlap.

A *shard* is a list of ``(l, r, w)`` triples, one per dimension: the rank holds indices
``[l, r)`` of a dimension of width ``w``.  Two ranks may describe the same logical tensor
with different factorisations (a flat ``[24]`` versus ``[4, 6]`` versus ``[2, 3, 4]``); the
alignment below builds their common refinement so the boxes can be intersected.

Parity with the reference (``wbridge/utils/data.py``):

* ``WeightData`` keeps the reference's metadata format and API
  (``data.py:63-201``: ``meta_dict``, ``to_jsonable``, ``__bytes__``, ``iter_with_intv``,
  ``total_nbytes``, ``compute_overlap``), with a multi-shard entry treated as a disjoint
  union whose byte size is the sum over its shards (the reference counts only the first
  shard, ``data.py:53-54,159-164``) and without the equal-numel restriction on shards.
* ``check_shard_compatibility`` returns the pair form ``(aligned_s, aligned_r)`` that the
  reference's tests expect (``tests/test_shard_compatibility.py:35-303``); the 5-tuple form
  of ``data.py:323-384`` is ``align_shards``.  The refinement rules are the ones the tests
  pin down: a dimension ``(l*a, r*a, w*a)`` equals ``[(l, r, w), (0, a, a)]``, and a range
  inside one row of the outer factor splits into ``(row, row+1) x (l', r')``.
* ``pack_for`` / ``tensors_from_flat`` are the round-trip API the reference's tests call
  (``tests/test_shard_compatibility.py:337-347``) but the reference never defined.

Each refined dimension also carries an element stride, so that the planner can turn an
overlap straight into a strided copy between two physical tensors (which may be strided
views into fused buffers such as a grouped QKV weight).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass
from typing import Any, Iterator, Sequence

import torch

from ..utils.dtypes import as_dtype, dtype_to_str

Triple = tuple[int, int, int]
Shard = list[Triple]
Shards = list[Shard]


# --------------------------------------------------------------------------------------
# shard helpers
# --------------------------------------------------------------------------------------

def _triple(t: Sequence[int]) -> Triple:
    if len(t) != 3:
        raise ValueError(f"shard dimension must be (l, r, w), got {t!r}")
    return (int(t[0]), int(t[1]), int(t[2]))


def normalize_shards(spec: Any) -> Shards:
    """Return the multi-shard form ``[[(l, r, w), ...], ...]`` of a single or multi shard."""
    if spec is None or len(spec) == 0:
        return []
    first = spec[0]
    if len(first) > 0 and not isinstance(first[0], (list, tuple)):
        return [[_triple(t) for t in spec]]
    return [[_triple(t) for t in shard] for shard in spec]


def shard_numel(shard: Shard) -> int:
    return math.prod(r - l for l, r, _ in shard)


def shard_extents(shard: Shard) -> list[int]:
    return [r - l for l, r, _ in shard]


def contiguous_strides(extents: Sequence[int]) -> list[int]:
    strides = [1] * len(extents)
    acc = 1
    for i in range(len(extents) - 1, -1, -1):
        strides[i] = acc
        acc *= max(int(extents[i]), 1)
    return strides


def original_total_numel(shards: Shards) -> int:
    """Elements held by an entry: the sum over its (disjoint) shards."""
    return sum(shard_numel(s) for s in shards)


def shards_iterator(shards: Shards, offset: int = 0, item_size: int = 1) -> Iterator[tuple[int, int, Shard]]:
    """Yield ``(start, end, shard)`` byte intervals of each shard in a packed entry."""
    for shard in shards:
        n = shard_numel(shard) * item_size
        yield offset, offset + n, shard
        offset += n


# --------------------------------------------------------------------------------------
# alignment (common refinement of two factorisations)
# --------------------------------------------------------------------------------------

@dataclass(frozen=True)
class Dim:
    """One dimension of a box: range ``[l, r)`` of width ``w``; ``stride`` in elements."""
    l: int
    r: int
    w: int
    stride: int = 0


@dataclass(frozen=True)
class AlignedDim:
    """One dimension of a common refinement: sender range, receiver range, shared width."""
    s: Dim
    r: Dim

    @property
    def w(self) -> int:
        return self.s.w


def _split_dim(d: Dim, outer_w: int) -> tuple[Dim, Dim] | None:
    """Factor ``d`` (width ``outer_w * tail``) into an outer dim of width ``outer_w`` and an
    inner dim of width ``tail``; ``None`` if ``[l, r)`` is not a rectangle in that grid."""
    tail = d.w // outer_w
    if d.l % tail == 0 and d.r % tail == 0:           # whole rows of the inner factor
        return (Dim(d.l // tail, d.r // tail, outer_w, d.stride * tail),
                Dim(0, tail, tail, d.stride))
    row = d.l // tail
    if (d.r - 1) // tail == row:                       # a run inside one row
        return (Dim(row, row + 1, outer_w, d.stride * tail),
                Dim(d.l - row * tail, d.r - row * tail, tail, d.stride))
    return None


def refine(a: Sequence[Dim], b: Sequence[Dim]) -> list[AlignedDim] | None:
    """Common refinement of two boxes over the same logical tensor, or ``None``.

    Walks both dimension lists from the outermost dimension inwards.  Where the current
    widths differ, the wider dimension must be a multiple of the narrower one and is
    factored as ``narrower x tail``; the tail factor stays current on that side.  Trailing
    width-1 dimensions on either side are absorbed.
    """
    ia, ib = iter(a), iter(b)
    ca, cb = next(ia, None), next(ib, None)
    out: list[AlignedDim] = []
    while ca is not None and cb is not None:
        if ca.w == cb.w:
            out.append(AlignedDim(ca, cb))
            ca, cb = next(ia, None), next(ib, None)
        elif ca.w > cb.w:
            if cb.w <= 0 or ca.w % cb.w:
                return None
            parts = _split_dim(ca, cb.w)
            if parts is None:
                return None
            out.append(AlignedDim(parts[0], cb))
            ca, cb = parts[1], next(ib, None)
        else:
            if ca.w <= 0 or cb.w % ca.w:
                return None
            parts = _split_dim(cb, ca.w)
            if parts is None:
                return None
            out.append(AlignedDim(ca, parts[0]))
            ca, cb = next(ia, None), parts[1]
    while ca is not None and ca.w == 1:
        out.append(AlignedDim(ca, Dim(0, 1, 1, 0)))
        ca = next(ia, None)
    while cb is not None and cb.w == 1:
        out.append(AlignedDim(Dim(0, 1, 1, 0), cb))
        cb = next(ib, None)
    if ca is not None or cb is not None:
        return None
    return out


def _dims(shard: Shard, strides: Sequence[int] | None = None) -> list[Dim]:
    if strides is None:
        strides = contiguous_strides(shard_extents(shard))
    if len(strides) != len(shard):
        raise ValueError(f"{len(strides)} strides for a {len(shard)}-d shard")
    return [Dim(l, r, w, int(st)) for (l, r, w), st in zip(shard, strides)]


def align_shards(s_shard: Shard, r_shard: Shard) -> list[tuple[int, int, int, int, int]] | None:
    """5-tuple form ``(l_s, r_s, l_r, r_r, w)`` per refined dimension, or ``None``."""
    al = refine(_dims(s_shard), _dims(r_shard))
    if al is None:
        return None
    return [(d.s.l, d.s.r, d.r.l, d.r.r, d.w) for d in al]


def check_shard_compatibility(s_shard: Shard, r_shard: Shard) -> tuple[Shard, Shard] | None:
    """Pair form ``(aligned_s, aligned_r)`` of the common refinement, or ``None``."""
    al = refine(_dims(normalize_shards(s_shard)[0]), _dims(normalize_shards(r_shard)[0]))
    if al is None:
        return None
    return ([(d.s.l, d.s.r, d.w) for d in al], [(d.r.l, d.r.r, d.w) for d in al])


# Reference name for the same check (pair form).
_check_shard_compatibility = check_shard_compatibility


@dataclass
class BoxCopy:
    """A strided copy between two bound boxes: offsets/strides in elements."""
    src_offset: int
    dst_offset: int
    extents: list[int]
    src_strides: list[int]
    dst_strides: list[int]
    # the intersected region in refined logical coordinates
    region: list[Triple]

    @property
    def numel(self) -> int:
        return math.prod(self.extents)


def box_copy(src_shard: Shard, dst_shard: Shard,
             src_strides: Sequence[int] | None = None,
             dst_strides: Sequence[int] | None = None) -> BoxCopy | None:
    """Intersect two boxes and express the intersection as a strided copy.

    Raises ``ValueError`` when the two factorisations cannot be aligned; returns ``None``
    when the boxes do not intersect.
    """
    al = refine(_dims(src_shard, src_strides), _dims(dst_shard, dst_strides))
    if al is None:
        raise ValueError(f"shards {src_shard} and {dst_shard} cannot be aligned")
    src_off = dst_off = 0
    ext, ss, ds, region = [], [], [], []
    for d in al:
        lo, hi = max(d.s.l, d.r.l), min(d.s.r, d.r.r)
        if lo >= hi:
            return None
        src_off += (lo - d.s.l) * d.s.stride
        dst_off += (lo - d.r.l) * d.r.stride
        ext.append(hi - lo)
        ss.append(d.s.stride)
        ds.append(d.r.stride)
        region.append((lo, hi, d.w))
    return BoxCopy(src_off, dst_off, ext, ss, ds, region)


def _logical_strides(shard: Shard) -> list[int]:
    """Elements of the logical tensor between consecutive indices of each box dimension."""
    out = [1] * len(shard)
    for d in range(len(shard) - 2, -1, -1):
        out[d] = out[d + 1] * int(shard[d + 1][2])
    return out


def _cut_sizes(shard: Shard, other: Shard) -> list[list[int]]:
    """Per dimension of ``shard``: the block sizes (in units of that dimension, largest first)
    of ``other``'s dimensions nested inside it, i.e. where ``other``'s factorisation puts
    boundaries that a range of this dimension may have to be cut at."""
    L, M = _logical_strides(shard), _logical_strides(other)
    out = []
    for (_l, _r, w), li in zip(shard, L):
        out.append(sorted({m // li for m in M if m % li == 0 and li < m < li * int(w)}, reverse=True))
    return out


def _split_range(l: int, r: int, sizes: Sequence[int]) -> list[tuple[int, int]]:
    """Cut ``[l, r)`` into pieces that are whole blocks of ``sizes[0]`` or lie inside one such
    block, recursively for the smaller sizes."""
    if not sizes:
        return [(l, r)]
    q, rest = sizes[0], sizes[1:]
    a, b = -(-l // q) * q, (r // q) * q
    if a >= b:
        if l // q == (r - 1) // q:
            return _split_range(l, r, rest)
        return _split_range(l, a, rest) + _split_range(a, r, rest)
    out = _split_range(l, a, rest) if l < a else []
    out.append((a, b))
    if b < r:
        out += _split_range(b, r, rest)
    return out


def _pieces(shard: Shard, strides: Sequence[int], other: Shard):
    """``(piece, element offset)`` of ``shard`` cut so that each piece aligns with ``other``."""
    import itertools
    per_dim = [_split_range(int(l), int(r), q) for (l, r, _w), q in zip(shard, _cut_sizes(shard, other))]
    for combo in itertools.product(*per_dim):
        off = sum((a - int(l)) * int(st) for (a, _b), (l, _r, _w), st in zip(combo, shard, strides))
        yield [(a, b, int(w)) for (a, b), (_l, _r, w) in zip(combo, shard)], off


def box_copies(src_shard: Shard, dst_shard: Shard,
               src_strides: Sequence[int] | None = None,
               dst_strides: Sequence[int] | None = None) -> list[BoxCopy]:
    """The intersection of two boxes as strided copies: one when the two factorisations
    align, else one per pair of aligned pieces.  A range that cuts through a block of the
    other side's refinement (an FSDP row range ending inside an attention head, against a
    per-head box) is cut at those block boundaries first, then, if needed, into runs with every
    leading index fixed; the pieces are rectangles in the common refinement.  Raises
    ``ValueError`` when the two boxes' dimensions are not refinements of one shape (4 x 6
    against 6 x 4: most likely a transposed or mis-declared tensor) or the pieces do not align."""
    try:
        bc = box_copy(src_shard, dst_shard, src_strides, dst_strides)
        return [] if bc is None else [bc]
    except ValueError:
        pass
    if not _nested(src_shard, dst_shard):
        raise ValueError(f"shards {src_shard} and {dst_shard} cannot be aligned: their dimensions are not "
                         "refinements of one shape (a transposed or mis-declared tensor?)")
    ss = list(src_strides) if src_strides is not None else contiguous_strides(shard_extents(src_shard))
    ds = list(dst_strides) if dst_strides is not None else contiguous_strides(shard_extents(dst_shard))
    try:
        return _cut_copies(src_shard, ss, dst_shard, ds)
    except ValueError:
        pass
    out = []
    for run, roff in _runs(src_shard, ss):
        try:
            got = _cut_copies(run, ss, dst_shard, ds)
        except ValueError:
            raise ValueError(f"shards {src_shard} and {dst_shard} cannot be aligned") from None
        for bc in got:
            bc.src_offset += roff
        out += got
    return out


def _nested(a: Shard, b: Shard) -> bool:
    """Whether two boxes' dimensions are refinements of one shape: the logical extents of all
    their dimension suffixes form a chain under divisibility (4 x 6 and 2 x 2 x 6 do; 4 x 6
    and 6 x 4 of the same 24 elements do not)."""
    pts = set()
    for box in (a, b):
        m = 1
        for _l, _r, w in reversed(box):
            m *= int(w)
            pts.add(m)
    pts = sorted(pts)
    return all(y % x == 0 for x, y in zip(pts, pts[1:]))


def _cut_copies(src_shard: Shard, ss: Sequence[int], dst_shard: Shard, ds: Sequence[int]) -> list[BoxCopy]:
    out = []
    dst_pieces = list(_pieces(dst_shard, ds, src_shard))
    for sp, soff in _pieces(src_shard, ss, dst_shard):
        for dp, doff in dst_pieces:
            bc = box_copy(sp, dp, ss, ds)
            if bc is not None:
                bc.src_offset += soff
                bc.dst_offset += doff
                out.append(bc)
    return out


def _runs(shard: Shard, strides: Sequence[int]):
    """``(run, element offset)``: ``shard`` cut into boxes whose dims before the first one
    that is followed only by whole dims are single indices (logically contiguous runs)."""
    import itertools
    k = len(shard) - 1
    while k > 0 and all(int(l) == 0 and int(r) == int(w) for l, r, w in shard[k:]):
        k -= 1
    prefix = [range(int(l), int(r)) for l, r, _w in shard[:k]]
    for idx in itertools.product(*prefix):
        off = sum((i - int(l)) * int(st) for i, (l, _r, _w), st in zip(idx, shard, strides))
        yield [(i, i + 1, int(w)) for i, (_l, _r, w) in zip(idx, shard)] + [tuple(int(x) for x in d) for d in shard[k:]], off


def _drop_contained(boxes: list[Shard]) -> list[Shard]:
    """The regions not contained in another one (of identical ones, the first).  A receiver
    entry whose shards overlap (redundant expert slots, MLA's ``w_kc`` / ``w_vc`` inside
    ``kv_b_proj``) would otherwise carry the shared elements once per shard; the receiver
    writes a region into every shard it intersects, so one copy is enough."""
    keep = []
    for i, a in enumerate(boxes):
        na = shard_numel(a)
        inside = False
        for j, b in enumerate(boxes):
            if i == j:
                continue
            nb = shard_numel(b)
            if nb < na or (nb == na and j > i):
                continue
            try:
                k = sum(bc.numel for bc in box_copies(a, b))
            except ValueError:
                continue
            if k == na:
                inside = True
                break
        if not inside:
            keep.append(a)
    return keep


def covered_numel(region: Shard, shards: Sequence[Shard]) -> int:
    """Elements of ``shards`` (counted once per shard) that ``region`` fills."""
    return sum(bc.numel for rs in shards for bc in box_copies(region, rs))


def scale_box(region: Shard, block: Sequence[int], name: str = "") -> Shard:
    """Block-scale cells a 2-D region of a quantised tensor touches.  A cell of a block the
    region only partly covers is shared with the other senders of that block (they all
    write the same scale, see ``core/splitq.py``)."""
    if len(region) > 2:          # a refined row dimension: the logical rows it covers
        from .splitq import region_rows
        region = [region_rows(region), region[-1]]
    if len(region) != 2:
        raise ValueError(f"{name}: a block-quantised overlap needs rows and columns, got {region}")
    return [(l // b, (r + b - 1) // b, (w + b - 1) // b) for (l, r, w), b in zip(region, block)]


def coalesce(extents: Sequence[int], src_strides: Sequence[int], dst_strides: Sequence[int]
             ) -> tuple[list[int], list[int], list[int]]:
    """Drop extent-1 dims and merge neighbours that are contiguous on both sides."""
    e, s, d = [], [], []
    for x, a, b in zip(extents, src_strides, dst_strides):
        if x != 1:
            e.append(int(x)); s.append(int(a)); d.append(int(b))
    if not e:
        return [1], [1], [1]
    i = len(e) - 2
    while i >= 0:
        if s[i] == e[i + 1] * s[i + 1] and d[i] == e[i + 1] * d[i + 1]:
            e[i + 1] *= e[i]
            del e[i], s[i], d[i]
        i -= 1
    return e, s, d


# --------------------------------------------------------------------------------------
# WeightData
# --------------------------------------------------------------------------------------

class WeightData:
    """Shard metadata for weight transfer (no tensor storage).

    ``meta_dict`` maps a logical tensor name to ``{"shard": [[(l, r, w), ...], ...],
    "dtype": torch.dtype}`` plus optional keys: ``"quant"`` (a receiver that stores the
    tensor quantized, e.g. ``{"format": "fp8_block", "block": [128, 128], "scale":
    "<name of the fp32 scale tensor>"}``) and ``"src_dtype"`` (on an overlap whose two
    sides differ in dtype).  Shards are kept in the multi-shard form; a single shard
    ``[(l, r, w), ...]`` is accepted on input.  ``dtype`` may be given as a string.
    """

    def __init__(self, meta_dict: dict[str, dict[str, Any]] | bytes | str | None = None):
        if meta_dict is None:
            meta_dict = {}
        if isinstance(meta_dict, (bytes, bytearray)):
            meta_dict = meta_dict.decode("utf-8")
        if isinstance(meta_dict, str):
            meta_dict = json.loads(meta_dict)
        self.meta_dict: dict[str, dict[str, Any]] = {}
        for name, value in meta_dict.items():
            self.meta_dict[name] = self._normalize_entry(name, value)

    @staticmethod
    def _normalize_entry(name: str, value: dict[str, Any]) -> dict[str, Any]:
        shards = normalize_shards(value["shard"])
        if not shards:
            raise ValueError(f"empty shard list for {name}")
        for shard in shards:
            if not shard:
                raise ValueError(f"empty shard in list for {name}")
            for l, r, w in shard:
                if not (0 <= l < r <= w):
                    raise ValueError(f"invalid shard dim {(l, r, w)} for {name}")
        entry = {"shard": shards, "dtype": as_dtype(value["dtype"])}
        for key in ("quant", "src_dtype"):
            if value.get(key) is not None:
                entry[key] = as_dtype(value[key]) if key == "src_dtype" else dict(value[key])
        return entry

    # -- container protocol ---------------------------------------------------------
    def __iter__(self) -> Iterator[tuple[str, Shards, torch.dtype]]:
        for name, e in self.meta_dict.items():
            yield name, e["shard"], e["dtype"]

    def __len__(self) -> int:
        return len(self.meta_dict)

    def __bool__(self) -> bool:
        return bool(self.meta_dict)

    def __contains__(self, name: str) -> bool:
        return name in self.meta_dict

    def __getitem__(self, name: str) -> dict[str, Any]:
        """Entry of ``name``; a one-shard entry shows its shard in the single-shard form."""
        e = dict(self.meta_dict[name])
        if len(e["shard"]) == 1:
            e["shard"] = list(e["shard"][0])
        return e

    def __setitem__(self, name: str, value: dict[str, Any]) -> None:
        self.meta_dict[name] = self._normalize_entry(name, value)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, WeightData) and self.to_jsonable() == other.to_jsonable()

    def names(self) -> list[str]:
        return list(self.meta_dict)

    def shards(self, name: str) -> Shards:
        return self.meta_dict[name]["shard"]

    def dtype(self, name: str) -> torch.dtype:
        return self.meta_dict[name]["dtype"]

    def quant(self, name: str) -> dict[str, Any] | None:
        return self.meta_dict[name].get("quant")

    def numel(self, name: str) -> int:
        return original_total_numel(self.shards(name))

    # -- serialisation -------------------------------------------------------------
    def to_jsonable(self) -> dict[str, dict[str, Any]]:
        out: dict[str, dict[str, Any]] = {}
        for name, e in self.meta_dict.items():
            j: dict[str, Any] = {"shard": [[list(t) for t in s] for s in e["shard"]],
                                 "dtype": dtype_to_str(e["dtype"])}
            if "quant" in e:
                j["quant"] = e["quant"]
            if "src_dtype" in e:
                j["src_dtype"] = dtype_to_str(e["src_dtype"])
            out[name] = j
        return out

    def __str__(self) -> str:
        return json.dumps(self.to_jsonable(), separators=(",", ":"))

    def __repr__(self) -> str:
        return f"WeightData({len(self)} entries, {self.total_nbytes()} bytes)"

    def __bytes__(self) -> bytes:
        return str(self).encode("utf-8")

    # -- byte accounting -----------------------------------------------------------
    def iter_with_intv(self) -> Iterator[tuple[int, int, str, Shards, torch.dtype]]:
        """Yield ``(start, end, name, shards, dtype)`` of each entry in the packed layout."""
        off = 0
        for name, shards, dtype in self:
            n = original_total_numel(shards) * dtype.itemsize
            yield off, off + n, name, shards, dtype
            off += n

    def total_nbytes(self) -> int:
        return sum(original_total_numel(s) * dt.itemsize for _, s, dt in self)

    # -- overlap ---------------------------------------------------------------------
    @staticmethod
    def compute_overlap(sender: "WeightData", receiver: "WeightData") -> "WeightData":
        """Regions where ``sender`` and ``receiver`` overlap, in refined coordinates.

        Every sender shard is intersected with every receiver shard of the same name.
        The overlap entry's dtype is the sender's (the bytes on the wire); if the receiver
        stores another dtype it is recorded as the entry's conversion target.
        """
        result: dict[str, dict[str, Any]] = {}
        for name, s_shards, s_dtype in sender:
            if name not in receiver:
                continue
            r_dtype = receiver.dtype(name)
            boxes: Shards = []
            for ss in s_shards:
                for rs in receiver.shards(name):
                    try:
                        bcs = box_copies(ss, rs)
                    except ValueError as e:
                        raise ValueError(f"shard compatibility check failed for {name}: {e}") from None
                    boxes += [bc.region for bc in bcs]
            if len(receiver.shards(name)) > 1:
                boxes = _drop_contained(boxes)
            if boxes:
                entry: dict[str, Any] = {"shard": boxes, "dtype": s_dtype}
                if r_dtype != s_dtype:
                    entry = {"shard": boxes, "dtype": r_dtype, "src_dtype": s_dtype}
                    q = receiver.quant(name)
                    if q and q.get("format") == "fp8_block":
                        entry["quant"] = q
                        result[name] = entry
                        result[q["scale"]] = {
                            "shard": [scale_box(b, q["block"], name) for b in boxes],
                            "dtype": torch.float32, "quant": {"role": "scale", "of": name}}
                        continue
                result[name] = entry
        return WeightData(result)

    # -- host-side pack / unpack (reference-compatible convenience API) ---------------
    @staticmethod
    def pack_for(sender: "WeightData", tensors: dict[str, torch.Tensor],
                 overlap: "WeightData") -> torch.Tensor:
        """Pack the ``overlap`` regions of ``tensors`` (laid out as ``sender``) into one flat
        ``uint8`` buffer in ``overlap.iter_with_intv()`` order."""
        from .binding import bind, pack_into
        binding = bind(sender, tensors)
        first = next(iter(tensors.values()), None)
        device = first.device if first is not None else "cpu"
        out = torch.empty(overlap.total_nbytes(), dtype=torch.uint8, device=device)
        pack_into(binding, overlap, out)
        return out

    def tensors_from_flat(self, flat: torch.Tensor) -> dict[str, torch.Tensor]:
        """Split a packed buffer (``iter_with_intv`` layout) into typed per-entry tensors:
        the box's shape for a one-shard entry, 1-D for a multi-shard entry."""
        flat = flat.reshape(-1).view(torch.uint8)
        out: dict[str, torch.Tensor] = {}
        for start, end, name, shards, dtype in self.iter_with_intv():
            t = flat[start:end].view(dtype)
            out[name] = t.view(shard_extents(shards[0])) if len(shards) == 1 else t
        return out

    def __call__(self, tensors: dict[str, torch.Tensor]) -> "TensorBridge":
        """Bind ``tensors`` to this metadata: ``f[overlaps]`` packs, ``f[overlaps] = chunks``
        unpacks (``overlaps`` maps a peer rank to its overlap ``WeightData``)."""
        return TensorBridge(self, tensors)


class TensorBridge:
    """``metadata(tensors)``: overlap-indexed pack/unpack for the reference-compatible API.

    Unlike the reference (``data.py:219-238``), binding does not modify the caller's dict.
    """

    def __init__(self, metadata: WeightData, tensors: dict[str, torch.Tensor]):
        from .binding import bind
        self.metadata = metadata
        self.binding = bind(metadata, tensors)

    def __getitem__(self, dst_metas: dict[int, WeightData]) -> dict[int, torch.Tensor]:
        from .binding import pack_into
        out = {}
        for rank, ov in dst_metas.items():
            buf = torch.empty(ov.total_nbytes(), dtype=torch.uint8, device=self.binding.device)
            pack_into(self.binding, ov, buf)
            out[rank] = buf
        return out

    def __setitem__(self, src_metas: dict[int, WeightData],
                    chunks: dict[int, torch.Tensor] | torch.Tensor) -> None:
        from .binding import unpack_from
        if isinstance(chunks, torch.Tensor):
            if len(src_metas) != 1:
                raise ValueError("a single chunk needs exactly one overlap")
            chunks = {next(iter(src_metas)): chunks}
        for rank, ov in src_metas.items():
            unpack_from(self.binding, ov, chunks[rank])

