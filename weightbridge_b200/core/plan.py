"""Transfer planner: overlaps between bound shards -> strided ops -> flat device work tables.

A sender binds its local views (absolute addresses); a receiver publishes a *physical
binding*: for each entry shard, the allocation it lives in (an index into the receiver's
exported allocation table), the byte offset inside it and the element strides.  With
both, every overlap becomes one op:

* ``copy``  - same dtype, N-d strided copy (coalesced to as few dims as possible);
* ``cast``  - float -> float elementwise conversion (fp32 <-> bf16 <-> fp16);
* ``quant`` - a block-aligned 2-D region quantised to fp8 e4m3 with fp32 block scales
  written to the receiver's scale tensor;
* ``squant`` - one sender's part of a block that several senders share (``core/splitq.py``):
  quantised with the block amax the senders exchange before the launch.

Ops are lowered to the work tables the sm_100a kernel and the C++ CPU executor walk:
``ITEM`` rows (one 2-D copy/cast of at most ``item_bytes``) and ``QDESC`` rows (one
quantised matrix) with one ``QWORK`` row per 128x128 block.  The reference instead packs
each overlap into a wire buffer with one torch copy per box and sends it over NCCL
(``wbridge/utils/data.py:240-320``, ``wbridge/backend/direct_sender.py:184-198``).
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass, field
from typing import Callable, Iterable, Sequence

import numpy as np
import torch

from ..utils.dtypes import FLOAT_CAST_DTYPES, dtype_code, dtype_to_str
from .binding import Binding
from .shard import Shard, WeightData, box_copies, coalesce, contiguous_strides, shard_extents, shard_numel

# -- device table layouts (csrc/wb_common.h declares the same structs) ----------------------
ITEM_DTYPE = np.dtype([
    ("src", "<u8"), ("dst", "<u8"), ("src_pitch", "<i8"), ("dst_pitch", "<i8"),
    ("row_bytes", "<u4"), ("rows", "<u4"), ("op", "<u4"), ("dst_row_bytes", "<u4"),
])
QDESC_DTYPE = np.dtype([
    ("src", "<u8"), ("dst", "<u8"), ("scale", "<u8"), ("src_pitch", "<i8"), ("dst_pitch", "<i8"),
    ("scale_pitch", "<i8"), ("rows", "<u4"), ("cols", "<u4"), ("src_code", "<u4"),
    ("bn", "<u2"), ("bk", "<u2"),
])
QWORK_DTYPE = np.dtype([("desc", "<u4"), ("block", "<u4")])
SPIECE_DTYPE = np.dtype([
    ("src", "<u8"), ("dst", "<u8"), ("scale", "<u8"), ("src_pitch", "<i8"), ("dst_pitch", "<i8"),
    ("rows", "<u4"), ("cols", "<u4"), ("src_code", "<u4"), ("reserved", "<u4", (3,)),
])
assert ITEM_DTYPE.itemsize == 48 and QDESC_DTYPE.itemsize == 64 and QWORK_DTYPE.itemsize == 8
assert SPIECE_DTYPE.itemsize == 64

OP_COPY, OP_CAST, OP_COPY_MC, OP_TRANSPOSE = 0, 1, 2, 3
DEFAULT_ITEM_BYTES = 1 << 19


def op_word(kind: int, src: torch.dtype | None = None, dst: torch.dtype | None = None) -> int:
    w = kind
    if src is not None:
        w |= dtype_code(src) << 8
    if dst is not None:
        w |= dtype_code(dst) << 16
    return w


# -- physical bindings --------------------------------------------------------------------

@dataclass
class PhysShard:
    """Where one entry shard lives: allocation index (-1: ``offset`` is an absolute
    address in the current process), byte offset, element strides per box dim."""
    shard: Shard
    alloc: int
    offset: int
    strides: list[int]

    def to_json(self) -> list:
        return [[list(t) for t in self.shard], self.alloc, self.offset, list(self.strides)]

    @staticmethod
    def from_json(j) -> "PhysShard":
        return PhysShard([tuple(t) for t in j[0]], int(j[1]), int(j[2]), [int(s) for s in j[3]])


@dataclass
class PhysBinding:
    """Serializable description of a rank's bound tensors (address-level)."""
    meta: WeightData
    entries: dict[str, list[PhysShard]] = field(default_factory=dict)

    def to_json(self) -> dict:
        return {"meta": self.meta.to_jsonable(),
                "entries": {k: [p.to_json() for p in v] for k, v in self.entries.items()}}

    @staticmethod
    def from_json(j: dict) -> "PhysBinding":
        return PhysBinding(WeightData(j["meta"]),
                           {k: [PhysShard.from_json(p) for p in v] for k, v in j["entries"].items()})


def phys_binding(binding: Binding, locate: Callable[[int], tuple[int, int]] | None = None) -> PhysBinding:
    """Physical binding of a local ``Binding``.  ``locate(addr) -> (alloc, offset)`` maps a
    data pointer into an exported allocation table; without it addresses are absolute."""
    pb = PhysBinding(binding.meta)
    for name, views in binding.entries.items():
        lst = []
        for bs in views:
            addr = bs.tensor.data_ptr()
            alloc, off = locate(addr) if locate is not None else (-1, addr)
            lst.append(PhysShard(bs.shard, alloc, off, list(bs.strides)))
        pb.entries[name] = lst
    return pb


def wire_binding(overlap: WeightData, base: int = 0, alloc: int = -1) -> PhysBinding:
    """Physical binding of a packed wire buffer laid out in ``overlap.iter_with_intv()`` order."""
    pb = PhysBinding(overlap)
    for start, _e, name, shards, dtype in overlap.iter_with_intv():
        off = base + start
        lst = []
        for s in shards:
            lst.append(PhysShard(s, alloc, off, contiguous_strides(shard_extents(s))))
            off += shard_numel(s) * dtype.itemsize
        pb.entries[name] = lst
    return pb


# -- ops --------------------------------------------------------------------------------

@dataclass
class Op:
    kind: str                     # copy | cast | quant
    name: str
    src: tuple[int, int]          # (alloc, byte offset) on the source side
    dst: tuple[int, int]          # (alloc, byte offset) on the destination side
    extents: list[int]
    src_strides: list[int]        # elements
    dst_strides: list[int]
    src_dtype: torch.dtype
    dst_dtype: torch.dtype
    scale: tuple[int, int] | None = None      # quant: scale tensor start (alloc, byte offset)
    scale_strides: list[int] | None = None    # quant: element strides of the scale grid
    block: tuple[int, int] | None = None
    key: tuple | None = None                  # squant: (name, block row, block col) of the split block

    @property
    def src_bytes(self) -> int:
        return math.prod(self.extents) * self.src_dtype.itemsize

    @property
    def dst_bytes(self) -> int:
        n = math.prod(self.extents) * self.dst_dtype.itemsize
        if self.kind == "quant":
            bn, bk = self.block
            n += math.ceil(self.extents[0] / bn) * math.ceil(self.extents[1] / bk) * 4
        elif self.kind == "squant":
            n += 4
        return n


def _shift(p: PhysShard, nbytes: int) -> tuple[int, int]:
    return (p.alloc, p.offset + nbytes)


def plan_pair(src: PhysBinding, dst: PhysBinding, names: Iterable[str] | None = None,
              overlap_meta: WeightData | None = None) -> list[Op]:
    """All ops moving the overlap of ``src`` into ``dst`` (optionally restricted to ``names``).

    ``overlap_meta`` (when ``dst`` is a wire buffer) supplies quant specs and the scale
    entries of the overlap; otherwise they come from ``dst.meta``.
    """
    qsrc = overlap_meta if overlap_meta is not None else dst.meta
    ops: list[Op] = []
    wanted = set(names) if names is not None else None
    for name, s_shards, s_dtype in src.meta:
        if name not in dst.meta or (wanted is not None and name not in wanted):
            continue
        d_dtype = dst.meta.dtype(name)
        q = qsrc.quant(name) if name in qsrc else None
        quant = bool(q and q.get("format") == "fp8_block" and d_dtype != s_dtype)
        if not quant and d_dtype != s_dtype and not (s_dtype in FLOAT_CAST_DTYPES and d_dtype in FLOAT_CAST_DTYPES):
            raise TypeError(f"{name}: no conversion from {s_dtype} to {d_dtype}")
        for sp in src.entries[name]:
            for di, dp in enumerate(dst.entries[name]):
                try:
                    bcs = box_copies(sp.shard, dp.shard, sp.strides, dp.strides)
                except ValueError as e:
                    raise ValueError(f"shard compatibility check failed for {name}: {e}") from None
                for bc in bcs:
                    src_at = _shift(sp, bc.src_offset * s_dtype.itemsize)
                    dst_at = _shift(dp, bc.dst_offset * d_dtype.itemsize)
                    if quant:
                        ops += _quant_ops(name, q, bc, src_at, dst_at, s_dtype, d_dtype, dst, di)
                        continue
                    e, ss, ds = coalesce(bc.extents, bc.src_strides, bc.dst_strides)
                    ops.append(Op("copy" if s_dtype == d_dtype else "cast", name, src_at, dst_at, e, ss, ds,
                                  s_dtype, d_dtype))
    return ops


def _scale_cell(dst: PhysBinding, sname: str, name: str, bi: int, bj: int,
                shard: int | None = None) -> tuple[tuple[int, int], list[int]]:
    """(alloc, byte offset) of block (bi, bj)'s scale cell on the destination, and the scale
    grid's element strides.  When the scale entry has one shard per weight shard (always, for
    layouts with repeated shards such as redundant expert slots), the cell is taken from the
    weight shard's own scale shard ``shard``."""
    cands = dst.entries[sname]
    if shard is not None and len(cands) == len(dst.entries[name]):
        cands = [cands[shard]]
    for sp in cands:
        (a0, a1, _), (b0, b1, _) = sp.shard
        if a0 <= bi < a1 and b0 <= bj < b1:
            off = (bi - a0) * sp.strides[0] + (bj - b0) * sp.strides[1]
            return (sp.alloc, sp.offset + off * 4), list(sp.strides)
    raise ValueError(f"{name}: destination has no scale cell for block ({bi}, {bj})")


def _quant_ops(name, q, bc, src_at, dst_at, s_dtype, d_dtype, dst: PhysBinding, di: int | None = None) -> list[Op]:
    """The quantised ops of one overlap: per 2-D row sub-region (``core/splitq.py:
    row_subregions``; a refined row dimension such as Megatron's QKV groups gives several),
    its whole blocks as one ``quant`` op and one ``squant`` op per block it shares with other
    sub-regions or senders."""
    from .splitq import block_split, row_subregions
    if len(bc.extents) < 2:
        raise ValueError(f"{name}: a block-quantised overlap needs rows and columns, got {bc.region}")
    if bc.src_strides[-1] != 1 or bc.dst_strides[-1] != 1:
        raise ValueError(f"{name}: quantised rows must be contiguous on both sides")
    block = tuple(int(b) for b in q["block"])
    sname = q["scale"]
    se, de = s_dtype.itemsize, d_dtype.itemsize
    lows = [l for l, _r, _w in bc.region[:-2]]
    out = []
    for outer, rows, cols in row_subregions(bc.region):
        # element offsets of this sub-region's first row on both sides
        so = sum((i - l) * st for i, l, st in zip(outer, lows, bc.src_strides))
        do = sum((i - l) * st for i, l, st in zip(outer, lows, bc.dst_strides))
        src_sub = (src_at[0], src_at[1] + so * se)
        dst_sub = (dst_at[0], dst_at[1] + do * de)
        sst = [bc.src_strides[-2], bc.src_strides[-1]]
        dst_ = [bc.dst_strides[-2], bc.dst_strides[-1]]
        r0, c0 = rows[0], cols[0]
        core, pieces = block_split([rows, cols], block)

        def at(base, rr, cc, strides, es, r0=r0, c0=c0):
            return (base[0], base[1] + ((rr - r0) * strides[0] + (cc - c0) * strides[1]) * es)

        if core is not None:
            (cr0, cr1), (cc0, cc1) = core
            scale_at, sstr = _scale_cell(dst, sname, name, cr0 // block[0], cc0 // block[1], di)
            out.append(Op("quant", name, at(src_sub, cr0, cc0, sst, se), at(dst_sub, cr0, cc0, dst_, de),
                          [cr1 - cr0, cc1 - cc0], sst, dst_, s_dtype, d_dtype, scale_at, sstr, block))
        for (bi, bj), (pr0, pr1), (pc0, pc1) in pieces:
            scale_at, sstr = _scale_cell(dst, sname, name, bi, bj, di)
            out.append(Op("squant", name, at(src_sub, pr0, pc0, sst, se), at(dst_sub, pr0, pc0, dst_, de),
                          [pr1 - pr0, pc1 - pc0], sst, dst_, s_dtype, d_dtype, scale_at, sstr, block,
                          key=(name, bi, bj)))
    return out


def plan_digest(ops: Sequence[Op] | WeightData) -> str:
    """Hash of a plan's logical content; both sides compare it at connect."""
    if isinstance(ops, WeightData):
        payload = str(ops)
    else:
        payload = json.dumps([[o.kind, o.name, o.extents, dtype_to_str(o.src_dtype), dtype_to_str(o.dst_dtype)]
                              for o in ops])
    return hashlib.sha256(payload.encode()).hexdigest()[:16]


# -- lowering to device tables ------------------------------------------------------------

@dataclass
class Tables:
    items: np.ndarray                 # ITEM_DTYPE
    qdescs: np.ndarray                # QDESC_DTYPE
    qwork: np.ndarray                 # QWORK_DTYPE
    bytes_read: int = 0
    bytes_written: int = 0
    pieces: np.ndarray = field(default_factory=lambda: np.zeros(0, SPIECE_DTYPE))   # split-block parts
    piece_keys: list = field(default_factory=list)      # (receiver, name, bi, bj) per piece

    @staticmethod
    def empty() -> "Tables":
        return Tables(np.zeros(0, ITEM_DTYPE), np.zeros(0, QDESC_DTYPE), np.zeros(0, QWORK_DTYPE))

    @staticmethod
    def concat(ts: Sequence["Tables"]) -> "Tables":
        ts = list(ts)
        if not ts:
            return Tables.empty()
        qd, qw, off = [], [], 0
        for t in ts:
            qd.append(t.qdescs)
            w = t.qwork.copy()
            w["desc"] += off
            qw.append(w)
            off += len(t.qdescs)
        return Tables(np.concatenate([t.items for t in ts]), np.concatenate(qd), np.concatenate(qw),
                      sum(t.bytes_read for t in ts), sum(t.bytes_written for t in ts),
                      np.concatenate([t.pieces for t in ts]), [k for t in ts for k in t.piece_keys])

    def __len__(self) -> int:
        return len(self.items) + len(self.qwork) + len(self.pieces)


def _split_rows(src, dst, sp, dp, row_bytes, rows, op, drb, item_bytes, out: list):
    """Append items for ``rows`` rows of ``row_bytes`` (source bytes), at most ``item_bytes`` each."""
    if rows == 0 or row_bytes == 0:
        return
    dst_elem_ratio = drb / row_bytes if row_bytes else 1.0
    if row_bytes > item_bytes:
        # long rows: pieces along the row, aligned to 16 bytes on the source side
        piece = max(16, (item_bytes // 16) * 16)
        for r in range(rows):
            off = 0
            while off < row_bytes:
                n = min(piece, row_bytes - off)
                doff = int(off * dst_elem_ratio)
                dn = int(n * dst_elem_ratio)
                out.append((src + r * sp + off, dst + r * dp + doff, sp, dp, n, 1, op, dn))
                off += n
        return
    per = max(1, item_bytes // row_bytes)
    for r0 in range(0, rows, per):
        n = min(per, rows - r0)
        out.append((src + r0 * sp, dst + r0 * dp, sp, dp, row_bytes, n, op, drb))


def _lower_transpose(o: Op, s_addr: int, d_addr: int, ext, ss, ds, item_bytes: int, out: list) -> None:
    """Work rows of OP_TRANSPOSE for a copy whose last source dimension is contiguous and whose
    destination is contiguous along the second-to-last one: per outer index, R source rows by
    chunks of the C columns (``item_bytes`` of destination each, at least 64 columns)."""
    es = o.src_dtype.itemsize
    R, C = ext[-2], ext[-1]
    sp, dp = ss[-2] * es, ds[-1] * es
    word = op_word(OP_TRANSPOSE, o.src_dtype, o.dst_dtype)
    per = max(64, item_bytes // max(1, R * es))
    outer = ext[:-2]
    for idx in np.ndindex(*outer) if outer else [()]:
        so = sum(i * st for i, st in zip(idx, ss[:-2])) * es
        do = sum(i * st for i, st in zip(idx, ds[:-2])) * es
        for c0 in range(0, C, per):
            n = min(per, C - c0)
            out.append((s_addr + so + c0 * es, d_addr + do + c0 * dp, sp, dp, n * es, R, word, R * es))


def lower_ops(ops: Sequence[Op], src_base: Callable[[int], int], dst_base: Callable[[int], int],
              item_bytes: int = DEFAULT_ITEM_BYTES, multicast: bool = False, receiver: int = -1) -> Tables:
    """Resolve allocation indices to addresses and cut ops into device work rows.
    ``receiver`` prefixes the split-block keys of ``squant`` ops."""
    if item_bytes < 16:
        raise ValueError("item_bytes must be at least 16")
    item_bytes = min(int(item_bytes), 1 << 30)      # row_bytes / rows are 32-bit in the work rows
    items: list[tuple] = []
    qdescs: list[tuple] = []
    qwork: list[np.ndarray] = []
    pieces: list[tuple] = []
    keys: list[tuple] = []
    rd = wr = 0
    for o in ops:
        s_addr = src_base(o.src[0]) + o.src[1]
        d_addr = dst_base(o.dst[0]) + o.dst[1]
        se, de = o.src_dtype.itemsize, o.dst_dtype.itemsize
        rd += o.src_bytes
        wr += o.dst_bytes
        if o.kind == "quant":
            if multicast:
                raise ValueError(f"{o.name}: quantised blocks are stored per receiver, not multicast")
            rows, cols = o.extents
            bn, bk = o.block
            sc = dst_base(o.scale[0]) + o.scale[1]
            qdescs.append((s_addr, d_addr, sc, o.src_strides[0] * se, o.dst_strides[0] * de,
                           o.scale_strides[0] * 4, rows, cols, dtype_code(o.src_dtype), bn, bk))
            nb = math.ceil(rows / bn) * math.ceil(cols / bk)
            w = np.zeros(nb, QWORK_DTYPE)
            w["desc"] = len(qdescs) - 1
            w["block"] = np.arange(nb, dtype=np.uint32)
            qwork.append(w)
            continue
        if o.kind == "squant":
            if multicast:
                raise ValueError(f"{o.name}: quantised blocks are stored per receiver, not multicast")
            rows, cols = o.extents
            sc = dst_base(o.scale[0]) + o.scale[1]
            pieces.append((s_addr, d_addr, sc, o.src_strides[0] * se, o.dst_strides[0] * de, rows, cols,
                           dtype_code(o.src_dtype), (0, 0, 0)))
            keys.append((receiver,) + tuple(o.key))
            continue
        kind = OP_COPY if o.kind == "copy" else OP_CAST
        if multicast:
            if o.kind != "copy":
                raise ValueError(f"{o.name}: only same-dtype copies can be multicast, not {o.kind}")
            kind = OP_COPY_MC
        word = op_word(kind, o.src_dtype, o.dst_dtype)
        ext, ss, ds = list(o.extents), list(o.src_strides), list(o.dst_strides)
        if (kind == OP_COPY and len(ext) >= 2 and ss[-1] == 1 and ds[-1] != 1 and ds[-2] == 1
                and ext[-1] > 1 and ext[-2] > 1):
            # the destination is contiguous along the source's rows: tiled transposes (one
            # work row per outer index and column chunk) instead of one element per row
            _lower_transpose(o, s_addr, d_addr, ext, ss, ds, item_bytes, items)
            continue
        if ss[-1] == 1 and ds[-1] == 1:
            run = ext.pop()
            ss.pop(); ds.pop()
        else:
            run = 1
        rb, drb = run * se, run * de
        if not ext:
            _split_rows(s_addr, d_addr, rb, drb, rb, 1, word, drb, item_bytes, items)
            continue
        rows = ext[-1]
        sp, dp = ss[-1] * se, ds[-1] * de
        outer = ext[:-1]
        for idx in np.ndindex(*outer) if outer else [()]:
            so = sum(i * s for i, s in zip(idx, ss[:-1])) * se
            do = sum(i * s for i, s in zip(idx, ds[:-1])) * de
            _split_rows(s_addr + so, d_addr + do, sp, dp, rb, rows, word, drb, item_bytes, items)
    it = np.array(items, dtype=ITEM_DTYPE) if items else np.zeros(0, ITEM_DTYPE)
    qd = np.array(qdescs, dtype=QDESC_DTYPE) if qdescs else np.zeros(0, QDESC_DTYPE)
    qw = np.concatenate(qwork) if qwork else np.zeros(0, QWORK_DTYPE)
    pc = np.array(pieces, dtype=SPIECE_DTYPE) if pieces else np.zeros(0, SPIECE_DTYPE)
    return Tables(it, qd, qw, rd, wr, pc, keys)


# -- validation -----------------------------------------------------------------------------

def _code_bytes(code: int) -> int:
    from ..utils.dtypes import CODE_DTYPES
    dt = CODE_DTYPES.get(code)
    return dt.itemsize if dt is not None else 0


class PlanBoundsError(ValueError):
    """A work row would read or write outside the memory registered for it."""


def _merge(ranges: Sequence[tuple[int, int]]) -> tuple[np.ndarray, np.ndarray]:
    rs = sorted((int(a), int(b)) for a, b in ranges if b > a)
    lo, hi = [], []
    for a, b in rs:
        if lo and a <= hi[-1]:
            hi[-1] = max(hi[-1], b)
        else:
            lo.append(a)
            hi.append(b)
    return np.array(lo, dtype=np.uint64), np.array(hi, dtype=np.uint64)


def _check(starts: np.ndarray, ends: np.ndarray, ranges, what: str) -> None:
    if len(starts) == 0:
        return
    lo, hi = _merge(ranges)
    if len(lo) == 0:
        raise PlanBoundsError(f"{what}: no registered memory")
    idx = np.searchsorted(lo, starts, side="right").astype(np.int64) - 1
    ok = idx >= 0
    ok[ok] &= ends[ok] <= hi[idx[ok]]
    if not ok.all():
        bad = int(np.flatnonzero(~ok)[0])
        raise PlanBoundsError(f"{what}: row {bad} spans [{int(starts[bad]):#x}, {int(ends[bad]):#x}) outside "
                              f"every registered range")


def validate_tables(tables: Tables, src_ranges: Sequence[tuple[int, int]],
                    dst_ranges: Sequence[tuple[int, int]]) -> None:
    """Check every work row against the memory it may touch: reads inside ``src_ranges``
    (the sender's bound tensors), writes inside ``dst_ranges`` (the receivers' exported
    allocations).  Runs on the host before a table is uploaded, so a planning error is an
    exception rather than a stray store into another process's memory."""
    it = tables.items
    if len(it):
        rows = it["rows"].astype(np.uint64)
        last = np.maximum(rows, 1) - np.uint64(1)
        s0 = it["src"]
        s1 = s0 + last * it["src_pitch"].astype(np.uint64) + it["row_bytes"].astype(np.uint64)
        d0 = it["dst"]
        # a transpose writes one destination row per source column
        tp = (it["op"] & 0xFF) == OP_TRANSPOSE
        dlast = last.copy()
        if tp.any():
            es = np.array([max(1, _code_bytes(int(c))) for c in (it["op"][tp] >> 8) & 0xFF], dtype=np.uint64)
            dlast[tp] = np.maximum(it["row_bytes"][tp].astype(np.uint64) // es, 1) - np.uint64(1)
        d1 = d0 + dlast * it["dst_pitch"].astype(np.uint64) + it["dst_row_bytes"].astype(np.uint64)
        if (it["src_pitch"] < 0).any() or (it["dst_pitch"] < 0).any():
            raise PlanBoundsError("negative row pitch in a work row")
        _check(s0, s1, src_ranges, "read")
        _check(d0, d1, dst_ranges, "write")
    q = tables.qdescs
    if len(q):
        from ..utils.dtypes import CODE_DTYPES
        es = np.array([CODE_DTYPES[int(c)].itemsize for c in q["src_code"]], dtype=np.uint64)
        rows = q["rows"].astype(np.uint64)
        cols = q["cols"].astype(np.uint64)
        last = np.maximum(rows, 1) - np.uint64(1)
        _check(q["src"], q["src"] + last * q["src_pitch"].astype(np.uint64) + cols * es, src_ranges, "quant read")
        _check(q["dst"], q["dst"] + last * q["dst_pitch"].astype(np.uint64) + cols, dst_ranges, "quant write")
        bn, bk = q["bn"].astype(np.uint64), q["bk"].astype(np.uint64)
        nbr = (rows + bn - np.uint64(1)) // bn
        nbc = (cols + bk - np.uint64(1)) // bk
        _check(q["scale"], q["scale"] + (nbr - np.uint64(1)) * q["scale_pitch"].astype(np.uint64) + nbc * np.uint64(4),
               dst_ranges, "scale write")
    p = tables.pieces
    if len(p):
        from ..utils.dtypes import CODE_DTYPES
        if (p["src_pitch"] < 0).any() or (p["dst_pitch"] < 0).any():
            raise PlanBoundsError("negative row pitch in a split-block piece")
        es = np.array([CODE_DTYPES[int(c)].itemsize for c in p["src_code"]], dtype=np.uint64)
        last = np.maximum(p["rows"].astype(np.uint64), 1) - np.uint64(1)
        cols = p["cols"].astype(np.uint64)
        _check(p["src"], p["src"] + last * p["src_pitch"].astype(np.uint64) + cols * es, src_ranges, "piece read")
        _check(p["dst"], p["dst"] + last * p["dst_pitch"].astype(np.uint64) + cols, dst_ranges, "piece write")
        _check(p["scale"], p["scale"] + np.uint64(4), dst_ranges, "piece scale write")


def storage_ranges(tensors) -> list[tuple[int, int]]:
    """Byte ranges of the storages behind a collection of tensors (or lists of views)."""
    out = []
    for v in tensors:
        for t in (v if isinstance(v, (list, tuple)) else [v]):
            if isinstance(t, torch.Tensor):
                st = t.untyped_storage()
                out.append((st.data_ptr(), st.data_ptr() + st.nbytes()))
    return out


def multicast_ok(op: Op, src_base: Callable[[int], int], dst_base: Callable[[int], int]) -> bool:
    """Whether an op can go out as 16-byte multimem stores: a same-dtype copy whose rows
    start, end and stride on 16-byte boundaries on both sides."""
    if op.kind != "copy":
        return False
    es = op.src_dtype.itemsize
    if op.src_strides[-1] != 1 or op.dst_strides[-1] != 1:
        return False
    vals = [src_base(op.src[0]) + op.src[1], dst_base(op.dst[0]) + op.dst[1], op.extents[-1] * es]
    vals += [st * es for st in op.src_strides[:-1]] + [st * es for st in op.dst_strides[:-1]]
    return all(v % 16 == 0 for v in vals)
