"""Split fp8 blocks: 128 x 128 quantisation blocks whose elements come from several senders.

A block-quantised destination (``fp8_block``) has one fp32 scale per block, computed from the
amax of the whole block.  When the senders' shards cut through a block - a trainer with
expert TP whose FFN slice is not a multiple of 128 rows (Qwen3-30B-A3B experts, 768 rows, at
expert TP 4 hold 192 rows each), or dense TP slices such as 18944 / 8 = 2368 - no sender
holds the whole block.  Such a block is quantised in two steps:

1. every sender touching it reduces the amax of its part (one *piece* per block and shard);
2. the senders exchange their per-block maxima through the session (host), and each
   quantises its pieces with the common amax and writes the block's scale.

A region's blocks that lie entirely inside it form its *core* and go through the regular
quant path.  The reference never quantises (dtypes must match, ``wbridge/utils/data.py:181``).
"""
from __future__ import annotations

from typing import Iterable, Sequence

import numpy as np

from .shard import WeightData, box_copies

Region = Sequence[tuple[int, int, int]]          # [(l, r, w), (l, r, w)]
BlockKey = tuple                                 # (receiver, name, block row, block col)


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def _full_range(lo: int, hi: int, w: int, b: int) -> tuple[int, int]:
    """Block indices [first, last) whose whole extent lies inside [lo, hi) along one dim."""
    first = _cdiv(lo, b)
    last = _cdiv(w, b) if hi == w else hi // b
    return first, max(first, last)


def block_split(region: Region, block: Sequence[int]):
    """Split a 2-D region of a quantised tensor at its blocks.

    Returns ``(core, pieces)``: ``core`` is ``((r0, r1), (c0, c1))``, the sub-rectangle made of
    the blocks that lie entirely inside the region (``None`` if there are none), and
    ``pieces`` lists ``((bi, bj), (r0, r1), (c0, c1))`` for every other block the region
    touches, with the part of the block inside the region.  Block ``(bi, bj)`` spans rows
    ``[bi * bn, min((bi + 1) * bn, w_rows))`` of the logical tensor, and the same for columns.
    """
    (r0, r1, wr), (c0, c1, wc) = region
    bn, bk = int(block[0]), int(block[1])
    fr0, fr1 = _full_range(r0, r1, wr, bn)
    fc0, fc1 = _full_range(c0, c1, wc, bk)
    core = None
    if fr0 < fr1 and fc0 < fc1:
        core = ((fr0 * bn, min(fr1 * bn, wr)), (fc0 * bk, min(fc1 * bk, wc)))
    pieces = []
    for bi in range(r0 // bn, _cdiv(r1, bn)):
        for bj in range(c0 // bk, _cdiv(c1, bk)):
            if fr0 <= bi < fr1 and fc0 <= bj < fc1:
                continue
            pr = (max(r0, bi * bn), min(r1, (bi + 1) * bn))
            pc = (max(c0, bj * bk), min(c1, (bj + 1) * bk))
            pieces.append(((bi, bj), pr, pc))
    return core, pieces


def row_subregions(region: Region):
    """2-D pieces of a refined region of a 2-D logical tensor.

    The shard algebra may refine the row dimension into several (a Megatron QKV shard is
    ``[(groups), (rows per group), (cols)]``); a block-quantised op needs a uniform row pitch.
    Yields ``(outer, rows, cols)`` per index tuple ``outer`` of the refined row dims before the
    last one: ``rows = (l, r, W)`` in logical rows of the whole tensor, ``cols`` the last dim.
    A 2-D region yields itself with ``outer == ()``."""
    if len(region) < 2:
        raise ValueError(f"a block-quantised region needs rows and columns, got {region}")
    import itertools
    *rowdims, cols = [tuple(int(x) for x in d) for d in region]
    widths = [w for _l, _r, w in rowdims]
    W = 1
    for w in widths:
        W *= w
    inner_l, inner_r, inner_w = rowdims[-1]
    outer_dims = rowdims[:-1]
    for outer in itertools.product(*(range(l, r) for l, r, _w in outer_dims)):
        base, mult = 0, inner_w
        for idx, (_l, _r, w) in zip(reversed(outer), reversed(outer_dims)):
            base += idx * mult
            mult *= w
        yield outer, (base + inner_l, base + inner_r, W), cols


def region_rows(region: Region) -> tuple[int, int, int]:
    """The logical row range ``(l, r, W)`` a region covers; raises if it is not contiguous
    (the inner refined row dims must be whole)."""
    subs = list(row_subregions(region))
    lo, hi = subs[0][1][0], subs[-1][1][1]
    if sum(r - l for _o, (l, r, _w), _c in subs) != hi - lo:
        raise ValueError(f"region {region} covers non-contiguous rows of a block-quantised tensor")
    return lo, hi, subs[0][1][2]


def split_keys(sender: WeightData, receiver: WeightData, names: Iterable[str] | None = None) -> list[tuple]:
    """Sorted ``(name, bi, bj)`` of the split blocks ``sender`` sends to ``receiver``: the
    blocks of the receiver's quantised entries that the sender's regions touch without
    covering.  Depends only on metadata, so every sender can compute it for every other."""
    keys = set()
    wanted = set(names) if names is not None else None
    for name, s_shards, s_dtype in sender:
        if name not in receiver or (wanted is not None and name not in wanted):
            continue
        q = receiver.quant(name)
        if not (q and q.get("format") == "fp8_block" and receiver.dtype(name) != s_dtype):
            continue
        for ss in s_shards:
            for rs in receiver.shards(name):
                for bc in box_copies(ss, rs):
                    if len(bc.region) < 2:
                        continue
                    for _outer, rows, cols in row_subregions(bc.region):
                        for (bi, bj), _pr, _pc in block_split([rows, cols], q["block"])[1]:
                            keys.add((name, bi, bj))
    return sorted(keys)


class AmaxExchange:
    """Which split blocks this sender shares with which other senders, and how to merge
    their per-block maxima into its own.

    ``keys`` are this sender's split blocks ``(receiver, name, bi, bj)`` in the order its
    published maxima use; for every co-owner ``s``, ``pairs[s] = (mine, theirs)`` index the
    common blocks in this sender's and in ``s``'s order.
    """

    def __init__(self, rank: int, keys_by_sender: dict[int, list[tuple]]):
        self.rank = rank
        self.keys = keys_by_sender.get(rank, [])
        pos = {k: i for i, k in enumerate(self.keys)}
        self.pairs: dict[int, tuple[np.ndarray, np.ndarray]] = {}
        for s, ks in keys_by_sender.items():
            if s == rank or not ks:
                continue
            mine, theirs = [], []
            for j, k in enumerate(ks):
                i = pos.get(k)
                if i is not None:
                    mine.append(i)
                    theirs.append(j)
            if mine:
                self.pairs[s] = (np.array(mine, dtype=np.int64), np.array(theirs, dtype=np.int64))
        self.sizes = {s: len(ks) for s, ks in keys_by_sender.items()}

    @property
    def co_owners(self) -> list[int]:
        return sorted(self.pairs)

    def positions(self, piece_keys: Sequence[tuple]) -> np.ndarray:
        """Index of each piece's block in ``keys``."""
        pos = {k: i for i, k in enumerate(self.keys)}
        try:
            return np.array([pos[tuple(k)] for k in piece_keys], dtype=np.int64)
        except KeyError as e:
            raise ValueError(f"a piece of split block {e.args[0]} is missing from the exchange plan") from None

    def local(self, partial: np.ndarray, piece_pos: np.ndarray) -> np.ndarray:
        """Per-block maxima over this sender's own pieces."""
        vals = np.zeros(len(self.keys), dtype=np.float32)
        if len(piece_pos):
            np.maximum.at(vals, piece_pos, partial.astype(np.float32, copy=False))
        return vals

    def merge(self, vals: np.ndarray, others: dict[int, np.ndarray]) -> np.ndarray:
        out = vals.copy()
        for s, theirs_vals in others.items():
            mine, theirs = self.pairs[s]
            if len(theirs_vals) != self.sizes[s]:
                raise ValueError(f"sender {s} published {len(theirs_vals)} block maxima, expected {self.sizes[s]}")
            np.maximum.at(out, mine, theirs_vals[theirs])
        return out


def exchange_plan(rank: int, sender_metas: Sequence[WeightData], assignment: dict[int, dict[int, list[str]]],
                  receiver_metas: dict[int, WeightData]) -> AmaxExchange | None:
    """The amax exchange of ``rank``, or ``None`` when no receiver quantises anything."""
    if not any(any((m.quant(n) or {}).get("format") == "fp8_block" for n in m.names())
               for m in receiver_metas.values()):
        return None
    keys: dict[int, list[tuple]] = {}
    for s, targets in assignment.items():
        ks = []
        for r, names in sorted(targets.items()):
            if not names:
                continue
            ks += [(int(r),) + k for k in split_keys(sender_metas[int(s)], receiver_metas[int(r)], names)]
        keys[int(s)] = sorted(ks)
    return AmaxExchange(rank, keys)
